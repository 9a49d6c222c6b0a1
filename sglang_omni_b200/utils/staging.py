"""Pinned host staging buffers for per-step metadata uploads.

An engine step fills a pinned host buffer and enqueues its copy to the device
with ``non_blocking=True``; the copy runs when the stream reaches it, which
with overlapped scheduling is after the host has already started on the next
step.  A single buffer would then be rewritten before the queued copy read it,
and a step could run on the metadata of a later step (another batch bucket's
layout: out-of-range block-table rows).  ``PinnedRing`` hands out its buffers
round-robin and waits for the copy that last read a buffer before handing it
out again.
"""
from __future__ import annotations

import torch


class PinnedRing:
    def __init__(self, numel: int, dtype=torch.int32, n: int = 2, cuda: bool = True):
        self.cuda = cuda
        self.bufs = [torch.zeros(numel, dtype=dtype, pin_memory=cuda) for _ in range(n)]
        self.events: list = [None] * n
        self.i = 0

    def next(self) -> torch.Tensor:
        """The next buffer, free to overwrite."""
        self.i = (self.i + 1) % len(self.bufs)
        ev = self.events[self.i]
        if ev is not None:
            ev.synchronize()
            self.events[self.i] = None
        return self.bufs[self.i]

    @property
    def current(self) -> torch.Tensor:
        return self.bufs[self.i]

    def upload(self, dst: torch.Tensor, n: int, blocking: bool = False) -> None:
        """Copies the first ``n`` entries of the current buffer into ``dst`` on the current stream."""
        dst[:n].copy_(self.bufs[self.i][:n], non_blocking=not blocking)
        if self.cuda and not blocking:
            ev = torch.cuda.Event()
            ev.record()
            self.events[self.i] = ev
