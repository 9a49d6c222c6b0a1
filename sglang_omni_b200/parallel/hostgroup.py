"""Host-side bootstrap groups for the peer-memory kernels.

The fused TP / EP kernels move data over NVLink through symmetric buffers; the
host only has to exchange CUDA IPC handles once and meet at a few barriers.
``HostGroup`` does that over a ``torch.distributed.TCPStore`` without creating
a process group, so a stage's rank group can be formed inside a process that
already belongs to another group (the pipeline's NCCL relay group, a torchrun
job).  ``rank_of`` / ``world_of`` / ``all_gather_object`` / ``barrier`` accept
either a ``HostGroup`` or a ``torch.distributed`` group (``None`` = the default
group), which is what ``SymmetricBuffer``, ``TPGroup`` and ``EPMoE`` call.
"""
from __future__ import annotations

import pickle
from datetime import timedelta

import torch.distributed as dist


class HostGroup:
    def __init__(self, host: str, port: int, rank: int, world: int, timeout_s: float = 120.0,
                 prefix: str = "hg"):
        self.rank, self.world = rank, world
        self.prefix = prefix
        self.store = dist.TCPStore(host, port, world, rank == 0, timedelta(seconds=timeout_s),
                                   wait_for_workers=False)
        self._n = 0

    def subgroup(self, ranks: list[int], tag: str) -> "HostGroup":
        """A group of some of this group's ranks over the same store (call on those ranks only;
        ``tag`` distinguishes concurrent subgroups)."""
        sub = HostGroup.__new__(HostGroup)
        sub.rank, sub.world = list(ranks).index(self.rank), len(ranks)
        sub.prefix = f"{self.prefix}/{tag}"
        sub.store = self.store
        sub._n = 0
        return sub

    def _key(self, tag: str) -> str:
        return f"{self.prefix}/{self._n}/{tag}"

    def all_gather_object(self, obj) -> list:
        self._n += 1
        self.store.set(self._key(str(self.rank)), pickle.dumps(obj))
        out = [pickle.loads(self.store.get(self._key(str(r)))) for r in range(self.world)]
        self.barrier()
        return out

    def barrier(self) -> None:
        self._n += 1
        key = self._key("barrier")
        if int(self.store.add(key, 1)) == self.world:   # the last rank to arrive releases the others
            self.store.set(key + "/done", b"1")
        self.store.wait([key + "/done"])

    def broadcast_object(self, obj=None, src: int = 0):
        self._n += 1
        key = self._key("bcast")
        if self.rank == src:
            self.store.set(key, pickle.dumps(obj))
            return obj
        return pickle.loads(self.store.get(key))


def rank_of(group) -> int:
    return group.rank if isinstance(group, HostGroup) else dist.get_rank(group)


def world_of(group) -> int:
    return group.world if isinstance(group, HostGroup) else dist.get_world_size(group)


def all_gather_object(obj, group) -> list:
    if isinstance(group, HostGroup):
        return group.all_gather_object(obj)
    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out


def barrier(group) -> None:
    if isinstance(group, HostGroup):
        group.barrier()
    else:
        dist.barrier(group)
