"""NCCL point-to-point relay between stage processes (torch.distributed).

The sender posts ``isend`` on a dedicated CUDA stream and returns at once;
metadata carries the sender rank, byte count and a per-pair sequence tag so
the receiver posts the matching ``irecv`` into a buffer it allocates on its own
device.  Completion is read from a CUDA event (no host polling loop); every
wait is bounded.  Matches sglang_omni/relay/nccl.py:20-309 in behaviour
(explicit send / recv ranks, warm-up, 30 s bound).
"""
from __future__ import annotations

import asyncio
import os

import torch
import torch.distributed as dist

from .base import Relay, RelayOperation, register_relay


@register_relay("nccl")
class NcclRelay(Relay):
    def __init__(self, rank: int | None = None, world_size: int | None = None, device: str = "cuda",
                 group=None, **_):
        self.rank = rank if rank is not None else int(os.environ.get("RANK", "0"))
        self.world_size = world_size if world_size is not None else int(os.environ.get("WORLD_SIZE", "1"))
        self.device = torch.device(device if device != "cpu" else "cuda")
        self.group = group
        self._stream = None
        self._inflight: dict[str, list] = {}

    def warmup(self, peers) -> None:
        """Establishes the point-to-point connections with ``peers`` before the first transfer.
        NCCL sets a connection up on its first send / receive between two ranks, and the sender's
        host call blocks until the receiver has posted its side; a receiver that posts only after
        the sender's metadata arrives (which the sender publishes after its send call returns)
        would wait forever.  Collective over each pair: both ranks of every pair call this, with
        the pairs in one global order (``warmup_all``) so no rank waits on a pair its peer has not
        reached."""
        self._ensure()
        for peer in peers:
            if peer == self.rank:
                continue
            tx = torch.zeros(1, dtype=torch.uint8, device=self.device)
            rx = torch.empty(1, dtype=torch.uint8, device=self.device)
            ops = [dist.P2POp(dist.isend, tx, peer, group=self.group),
                   dist.P2POp(dist.irecv, rx, peer, group=self.group)]
            for w in dist.batch_isend_irecv(ops):
                w.wait()
        torch.cuda.synchronize(self.device)

    def warmup_all(self) -> None:
        """``warmup`` with every other rank of the group, pairs in ascending (low, high) order."""
        for a in range(self.world_size):
            for b in range(a + 1, self.world_size):
                if self.rank in (a, b):
                    self.warmup([b if self.rank == a else a])

    def _ensure(self):
        if not dist.is_initialized():
            raise RuntimeError("NcclRelay needs torch.distributed initialised (init_process_group('nccl'))")
        if self._stream is None:
            self._stream = torch.cuda.Stream(device=self.device)

    async def put_async(self, buffer, request_id, dst: int | None = None):
        self._ensure()
        buf = buffer.contiguous().view(torch.uint8).reshape(-1)
        if not buf.is_cuda:
            buf = buf.to(self.device, non_blocking=True)
        self._stream.wait_stream(torch.cuda.current_stream(self.device))
        ev = torch.cuda.Event()
        if dst is not None:
            with torch.cuda.stream(self._stream):
                work = dist.isend(buf, dst, group=self.group)
                work.wait()            # the side stream (not the host) waits for the send
            ev.record(self._stream)
            # the buffer stays referenced until the request is cleaned up
            self._inflight.setdefault(request_id, []).append((buf, work))
        return RelayOperation({"relay": "nccl", "src": self.rank, "nbytes": int(buf.numel())},
                              result=(buf, ev))

    async def get_async(self, metadata, dest=None):
        self._ensure()
        n = int(metadata["nbytes"])
        out = dest.view(torch.uint8).reshape(-1) if dest is not None else torch.empty(n, dtype=torch.uint8,
                                                                                       device=self.device)
        with torch.cuda.stream(self._stream):
            work = dist.irecv(out, int(metadata["src"]), group=self.group)
            work.wait()                # the side stream waits for the receive; the event marks its end
        ev = torch.cuda.Event()
        ev.record(self._stream)
        consumer = torch.cuda.current_stream(self.device)

        async def _wait():
            # bounded host poll of the event (30 s), then the consumer's stream is ordered after it
            for _ in range(300000):
                if ev.query():
                    consumer.wait_event(ev)
                    return out
                await asyncio.sleep(0.0001)
            raise TimeoutError("nccl relay receive timed out")

        return RelayOperation(metadata, future=asyncio.ensure_future(_wait()))

    def cleanup(self, request_id):
        self._inflight.pop(request_id, None)
