"""Loader of the sm_100a kernel extension and the per-device status word.

CUDA tensors always go through the extension: if it is missing on a machine
with a GPU, :func:`ext` raises instead of silently running a PyTorch fallback.
CPU tensors use the plain PyTorch restatements in each op module, which are
also the oracles of the kernel tests.
"""
from __future__ import annotations

import threading

import torch

_lock = threading.Lock()
_ext = None
_status: dict[int, torch.Tensor] = {}

STATUS_MESSAGES = {
    1: "mbarrier wait timed out inside a kernel",
    2: "peer flag wait timed out inside a fused collective kernel",
    3: "a kernel received an unsupported shape",
    4: "a device bounds check fired",
}


def ext():
    """Return the compiled ``sglang_omni_b200._C`` module or raise loudly."""
    global _ext
    if _ext is None:
        with _lock:
            if _ext is None:
                try:
                    from sglang_omni_b200 import _C  # type: ignore
                except ImportError as exc:  # pragma: no cover - depends on the build
                    raise RuntimeError(
                        "sglang_omni_b200._C is not built; run `python setup.py build_ext --inplace`"
                    ) from exc
                _ext = _C
    return _ext


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def status_word(device: torch.device) -> torch.Tensor:
    """int32 word the kernels of `device` write a non-zero code into on a bounded-wait timeout."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


def check_status(device: torch.device | None = None) -> None:
    """Synchronises and raises if any kernel on `device` recorded an error."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    t = status_word(device)
    code = int(t.item())
    if code != 0:
        t.zero_()
        msg = STATUS_MESSAGES.get(code)
        if msg is None and code >= 16:
            msg = f"mbarrier wait at site {code - 16} timed out inside a kernel"
        raise RuntimeError(f"device kernel error {code}: {msg or 'unknown'}")
