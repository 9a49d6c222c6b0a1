"""The shipped examples: the CPU one runs end to end, the GPU ones and the client compile, and the
two-GPU placement config validates against the schema."""
import os
import py_compile
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EX = os.path.join(ROOT, "examples")


def test_two_stage_toy_example_runs():
    r = subprocess.run([sys.executable, os.path.join(EX, "two_stage_toy.py")], capture_output=True, text=True,
                       timeout=600, cwd=ROOT, env=dict(os.environ, PYTHONPATH=ROOT))
    assert r.returncode == 0, r.stderr[-3000:]
    assert r.stdout.count("request ") == 4


def test_examples_compile():
    for f in os.listdir(EX):
        if f.endswith(".py"):
            py_compile.compile(os.path.join(EX, f), doraise=True)


def test_two_gpu_speech_config_validates():
    from sglang_omni_b200.config import ConfigManager

    cfg = ConfigManager.from_file(os.path.join(EX, "configs", "qwen3_omni_speech_2gpu.yaml"))
    assert cfg.gpu_placement["thinker"] == 0 and cfg.gpu_placement["talker_ar"] == 1
    assert cfg.relay_backend == "nccl"
    assert [s.name for s in cfg.stages][-2:] == ["talker_ar", "code2wav"]


def test_hf_llm_engine_example_runs():
    r = subprocess.run([sys.executable, os.path.join(EX, "hf_llm_engine.py"), "--tiny", "--device", "cpu",
                        "--max-new-tokens", "5"], capture_output=True, text=True, timeout=600, cwd=ROOT,
                       env=dict(os.environ, PYTHONPATH=ROOT))
    assert r.returncode == 0, r.stderr[-3000:]
    assert len(r.stdout.split()) == 5
