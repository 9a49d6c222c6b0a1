"""Symmetric device buffers: one allocation of the same size on every rank of a
group, each mapped into every peer process through CUDA IPC, so a kernel can
load from and store to any rank's copy over NVLink with plain pointers.

The table of base addresses (``peer_base``, int64 on the device) is what the
peer-memory kernels take; ``view`` gives a local torch view of a region.
"""
from __future__ import annotations

import torch

from ..ops._ext import ext
from .hostgroup import all_gather_object, barrier, rank_of, world_of


class SymmetricBuffer:
    def __init__(self, nbytes: int, group=None, device=None):
        self.group = group
        self.rank = rank_of(group)
        self.world = world_of(group)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.nbytes = int(nbytes)
        with torch.cuda.device(self.device):
            self.ptr = ext().ipc_alloc(self.nbytes)
            handle = ext().ipc_handle(self.ptr)
        handles = all_gather_object(handle, group)
        with torch.cuda.device(self.device):
            self.peers = [self.ptr if r == self.rank else ext().ipc_open(handles[r]) for r in range(self.world)]
        self.peer_base = torch.tensor(self.peers, dtype=torch.int64, device=self.device)
        barrier(group)
        self._closed = False

    def view(self, offset: int, shape, dtype) -> torch.Tensor:
        """Non-owning local view of [offset, offset + numel * itemsize)."""
        n = 1
        for d in shape:
            n *= int(d)
        assert offset + n * torch.empty(0, dtype=dtype).element_size() <= self.nbytes, "view outside the buffer"
        return ext().tensor_at(self.ptr + int(offset), [int(d) for d in shape], dtype, self.device.index)

    def close(self):
        """Collective: unmaps the peers' buffers and frees this rank's (after every rank is done with it)."""
        if self._closed:
            return
        torch.cuda.synchronize(self.device)
        barrier(self.group)
        with torch.cuda.device(self.device):
            for r, p in enumerate(self.peers):
                if r != self.rank:
                    ext().ipc_close(p)
        barrier(self.group)
        with torch.cuda.device(self.device):
            ext().ipc_free(self.ptr)
        self._closed = True


class RegionLayout:
    """Byte offsets of named regions inside a symmetric buffer (256-byte aligned)."""

    def __init__(self):
        self.offsets: dict[str, int] = {}
        self.size = 0

    def add(self, name: str, nbytes: int) -> int:
        off = (self.size + 255) // 256 * 256
        self.offsets[name] = off
        self.size = off + int(nbytes)
        return off
