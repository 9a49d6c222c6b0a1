"""Build of the native parts of sglang_omni_b200.

Two extensions, both built in-tree (``python setup.py build_ext --inplace``):

* ``sglang_omni_b200._C``        sm_100a CUDA kernels (tcgen05 / TMA / TMEM),
  compiled only for ``arch=compute_100a,code=sm_100a``;
* ``sglang_omni_b200._runtime``  host C++ runtime pieces (KV page allocator,
  batch metadata builder, shared-memory ring) that need no GPU.
"""
import glob
import os

from setuptools import setup

ROOT = os.path.dirname(os.path.abspath(__file__))
os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
os.environ.setdefault("MAX_JOBS", str(max(1, min(16, os.cpu_count() or 4))))

from torch.utils.cpp_extension import BuildExtension, CUDAExtension  # noqa: E402

CUDA_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("OMNI_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-DNDEBUG",
]
if os.environ.get("OMNI_DEVICE_CHECKS"):
    CUDA_FLAGS.append("-DOMNI_DEVICE_CHECKS=1")

cuda_sources = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + ["csrc/bindings.cpp"]
runtime_sources = sorted(glob.glob(os.path.join("csrc", "runtime", "*.cpp")))

ext_modules = [
    CUDAExtension(
        name="sglang_omni_b200._C",
        sources=cuda_sources,
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": CUDA_FLAGS},
    ),
]
if runtime_sources:
    # plain pybind11 module: no torch / CUDA linkage, importable on CPU-only hosts
    from pybind11.setup_helpers import Pybind11Extension

    ext_modules.append(
        Pybind11Extension(
            "sglang_omni_b200._runtime",
            sources=runtime_sources,
            include_dirs=[os.path.join(ROOT, "csrc", "runtime")],
            extra_compile_args=["-O3"],
            cxx_std=17,
            extra_link_args=["-lrt"],
        )
    )

setup(
    name="sglang_omni_b200",
    version="0.1.0",
    packages=["sglang_omni_b200"],
    package_data={"sglang_omni_b200": ["serve/playground.html"]},
    ext_modules=ext_modules,
    # the reference's command name (pyproject.toml:68 there): sgl-omni serve | config view | config export
    # sgl-omni-bench: the online serving benchmarks (tts-speed | omni-speed | tts-wer)
    entry_points={"console_scripts": ["sgl-omni=sglang_omni_b200.cli.cli:main",
                                      "sgl-omni-bench=sglang_omni_b200.benchmarks.__main__:main"]},
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
