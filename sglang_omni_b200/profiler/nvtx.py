"""NVTX ranges and CUDA-event device timers for stages, engine steps and
kernel families.  ``device_timer`` measures on the launching stream (events
recorded before and after, synchronised on read), the only timing this
project reports."""
from __future__ import annotations

import contextlib

import torch


@contextlib.contextmanager
def nvtx_range(name: str):
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class DeviceTimer:
    def __init__(self):
        self.events: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    @contextlib.contextmanager
    def time(self, name: str):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        try:
            yield
        finally:
            e.record()
            self.events.append((name, s, e))

    def summary(self) -> dict[str, float]:
        torch.cuda.synchronize()
        out: dict[str, float] = {}
        for n, s, e in self.events:
            out[n] = out.get(n, 0.0) + s.elapsed_time(e)
        return out
