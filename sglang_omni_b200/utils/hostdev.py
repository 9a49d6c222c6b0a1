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
