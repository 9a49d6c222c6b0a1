"""CPU shared-memory relay for stage processes on one host: one POSIX
shared-memory block per transfer, unlinked by the receiver; a credit pool
bounds blocks in flight (sglang_omni/relay/shm.py:18-181).  Device tensors
are staged through host memory."""
from __future__ import annotations

import asyncio
import uuid
from multiprocessing import shared_memory

import numpy as np
import torch

from .base import CreditAllocator, Relay, RelayOperation, register_relay


@register_relay("shm")
class ShmRelay(Relay):
    def __init__(self, credits: int = 2, device: str = "cpu", **_):
        self.device = device
        self.credits = CreditAllocator(max(credits, 64))
        self._owned: dict[str, list[shared_memory.SharedMemory]] = {}

    async def put_async(self, buffer, request_id):
        buf = buffer.detach().contiguous()
        if buf.is_cuda:
            buf = buf.cpu()
        data = buf.view(torch.uint8).numpy() if buf.dtype != torch.uint8 else buf.numpy()
        name = "omni_" + uuid.uuid4().hex[:24]
        shm = shared_memory.SharedMemory(name=name, create=True, size=max(1, data.nbytes))
        np.ndarray((data.nbytes,), dtype=np.uint8, buffer=shm.buf)[:] = data.reshape(-1)
        self._owned.setdefault(request_id, []).append(shm)
        shm.close()
        return RelayOperation({"relay": "shm", "name": name, "nbytes": int(data.nbytes)})

    async def get_async(self, metadata, dest=None):
        def _read():
            shm = shared_memory.SharedMemory(name=metadata["name"])
            try:
                arr = np.ndarray((metadata["nbytes"],), dtype=np.uint8, buffer=shm.buf).copy()
            finally:
                shm.close()
                shm.unlink()
            return torch.from_numpy(arr)

        t = await asyncio.to_thread(_read)
        if dest is not None:
            dest.view(torch.uint8).reshape(-1).copy_(t.to(dest.device))
            t = dest
        elif self.device != "cpu":
            t = t.to(self.device)
        return RelayOperation(metadata, result=t)

    def cleanup(self, request_id):
        self._owned.pop(request_id, None)
