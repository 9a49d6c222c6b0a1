"""Host -> device copies that never wait for the GPU.

A copy from pageable host memory (``torch.tensor(list, device=cuda)``,
``numpy_tensor.to(cuda)``) synchronises the stream before it starts.  When
several engine threads of one process share a stream, that wait includes all
the work the other threads have queued (a decode graph, a prefill), so
building a small index tensor can stall a thread for milliseconds.  ``h2d``
stages the data in pinned memory from PyTorch's caching host allocator and
copies with ``non_blocking=True``; the allocator keeps the pinned block alive
until the copy has run.
"""
from __future__ import annotations

import numpy as np
import torch


def h2d(data, device, dtype=None) -> torch.Tensor:
    """list / numpy array / CPU tensor -> tensor on ``device`` (asynchronous for CUDA)."""
    if isinstance(data, torch.Tensor):
        t = data if dtype is None else data.to(dtype)
    elif isinstance(data, np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(data))
        if dtype is not None:
            t = t.to(dtype)
    else:
        t = torch.tensor(data, dtype=dtype)
    device = torch.device(device)
    if device.type != "cuda":
        return t.to(device)
    if t.is_cuda:
        return t.to(device, non_blocking=True)
    if t.numel() == 0:
        return torch.empty(t.shape, dtype=t.dtype, device=device)
    return t.contiguous().pin_memory().to(device, non_blocking=True)


def own_stream(device) -> "torch.cuda.Stream | None":
    """A dedicated stream for one engine thread (None on CPU).  Engines of one
    process then only wait for their own queued work when they synchronise."""
    device = torch.device(device)
    if device.type != "cuda":
        return None
    return torch.cuda.Stream(device=device)


def adopt(t: torch.Tensor) -> torch.Tensor:
    """Marks a device tensor produced on another thread's stream as used on the
    current stream, so the allocator does not hand its memory back to the
    producer stream while this stream's queued work still reads it.  The data
    itself must already be complete (its producer synchronised, or the value
    is known to be finished through a host-side signal)."""
    if isinstance(t, torch.Tensor) and t.is_cuda:
        t.record_stream(torch.cuda.current_stream(t.device))
    return t
