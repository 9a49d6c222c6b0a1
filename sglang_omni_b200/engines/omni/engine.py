"""Generic step engine used by encoder stages (and any single-pass model):
schedule -> cache filter -> execute (worker thread for device work) -> cache
put -> update -> deliver, with one step in flight at a time.  Engine-step
failures fail every request of that batch only.

Reference counterpart: OmniEngine, sglang_omni/engines/omni/engine.py:34-612
(the autoregressive path lives in sglang_omni_b200.engines.ar).
"""
from __future__ import annotations

import asyncio
import logging
from typing import Any

import torch

from ..base import Engine
from .types import RequestOutput, SchedulerOutput

log = logging.getLogger(__name__)


class OmniEngine(Engine):
    def __init__(self, scheduler, model_runner, cache_manager=None, run_in_thread: bool = True,
                 stream_priority: int | None = None, poll_s: float = 0.0):
        """``stream_priority``: run steps on a dedicated CUDA stream of this priority
        (lower = served first by the block scheduler; encoders on the time-to-first-
        audio path use the highest).  ``poll_s``: sleep between polls while the
        planner holds requests back (a batching window)."""
        self.scheduler = scheduler
        self.model_runner = model_runner
        self.cache = cache_manager
        self.run_in_thread = run_in_thread
        self.stream_priority = stream_priority
        self.poll_s = poll_s
        self._stream = None
        self._task: asyncio.Task | None = None
        self._wake: asyncio.Event | None = None

    def _engine_stream(self):
        if self.stream_priority is None or self._stream is not None:
            return self._stream
        dev = torch.device(getattr(self.model_runner, "device", "cpu"))
        if dev.type == "cuda":
            self._stream = torch.cuda.Stream(device=dev, priority=self.stream_priority)
        return self._stream

    async def start(self):
        if self._task is None:
            self._wake = asyncio.Event()
            self._task = asyncio.ensure_future(self._run_loop())

    async def stop(self):
        if self._task is not None:
            self._task.cancel()
            self._task = None

    async def add_request(self, request_id: str, data: Any) -> None:
        await self.start()
        self.scheduler.add_request(request_id, data)
        self._wake.set()

    async def get_result(self, request_id: str) -> Any:
        return await self.scheduler.get_result(request_id)

    async def abort(self, request_id: str) -> None:
        self.scheduler.abort_request(request_id)

    def _filter_cached(self, sched_out: SchedulerOutput) -> dict[str, RequestOutput]:
        hits = {}
        if self.cache is None:
            return hits
        keep = []
        for r in sched_out.requests:
            v = self.cache.get(r)
            if v is not None:
                hits[r.request_id] = RequestOutput(r.request_id, v, finished=True)
            else:
                keep.append(r)
        if hits:
            sched_out.requests = keep
            sched_out.batch_data = self.scheduler.planner.build_batch(keep) if keep else None
        return hits

    async def _step(self, sched_out: SchedulerOutput) -> None:
        hits = self._filter_cached(sched_out)
        outputs: dict[str, RequestOutput] = dict(hits)
        reqs_all = list(sched_out.requests)
        if sched_out.requests:
            stream = self._engine_stream()
            if self.run_in_thread:
                res = await asyncio.to_thread(_execute_synced, self.model_runner, sched_out, stream)
            else:
                res = _execute_synced(self.model_runner, sched_out, stream)
            outputs.update(res.outputs)
            if self.cache is not None:
                for r in sched_out.requests:
                    o = res.outputs.get(r.request_id)
                    if o is not None and o.finished:
                        self.cache.put(r, o.data)
        # hits are delivered through the same update path
        sched_out.requests = reqs_all + [self.scheduler.requests[k] for k in hits if k in self.scheduler.requests
                                         and self.scheduler.requests[k] not in reqs_all]
        self.scheduler.update(sched_out, outputs)

    async def _run_loop(self):
        while True:
            sched_out = self.scheduler.schedule()
            if sched_out is None:
                self._wake.clear()
                if not self.scheduler.has_work():
                    await self._wake.wait()
                else:
                    await asyncio.sleep(self.poll_s)
                continue
            try:
                await self._step(sched_out)
            except asyncio.CancelledError:
                raise
            except Exception as exc:
                log.exception("engine step failed")
                self.scheduler.fail(sched_out, exc)


def _execute_synced(runner, sched_out, stream=None):
    """Runs one batch and waits for its GPU work: its output tensors go to other
    stages, whose threads run on their own streams."""
    if stream is not None:
        with torch.cuda.stream(stream):
            res = runner.execute(sched_out)
        stream.synchronize()
        return res
    res = runner.execute(sched_out)
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        torch.cuda.current_stream().synchronize()
    return res
