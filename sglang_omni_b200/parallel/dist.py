"""Process-group setup: one process per GPU, ``torch.distributed`` with NCCL
(gloo for CPU tests), rendezvous from the torchrun environment."""
from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist


@dataclass
class ParallelState:
    rank: int = 0
    world: int = 1
    local_rank: int = 0
    group: object = None

    @property
    def enabled(self) -> bool:
        return self.world > 1


def init_distributed(backend: str | None = None, timeout_s: float = 600.0) -> ParallelState:
    """Initialises the default process group from RANK / WORLD_SIZE / LOCAL_RANK (if more than one rank)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world <= 1:
        return ParallelState()
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if not dist.is_initialized():
        kw = {"timeout": timedelta(seconds=timeout_s)}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, **kw)
    return ParallelState(rank, world, local, dist.group.WORLD)
