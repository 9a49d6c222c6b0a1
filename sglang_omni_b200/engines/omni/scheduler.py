"""Request lifecycle scheduler of the generic step engine: WAITING -> RUNNING
(-> WAITING_FEEDBACK) -> FINISHED / ABORTED, delegating batch choice,
resources and iteration control; bounded retention of finished requests
(sglang_omni/engines/omni/scheduler.py:26-371)."""
from __future__ import annotations

import asyncio
import time
from collections import OrderedDict
from typing import Any

from .types import RequestOutput, SchedulerOutput, SchedulerRequest, SchedulerStatus


class Scheduler:
    def __init__(self, batch_planner, resource_manager, iteration_controller, max_retained: int = 10000):
        self.planner = batch_planner
        self.resources = resource_manager
        self.controller = iteration_controller
        self.waiting: list[SchedulerRequest] = []
        self.running: list[SchedulerRequest] = []
        self.requests: dict[str, SchedulerRequest] = {}
        self._results: dict[str, asyncio.Future] = {}
        self._streams: dict[str, asyncio.Queue] = {}
        self._finished: OrderedDict[str, Any] = OrderedDict()
        self.max_retained = max_retained
        self._step = 0

    def add_request(self, request_id: str, data: Any) -> None:
        req = SchedulerRequest(request_id, data)
        self.requests[request_id] = req
        self.waiting.append(req)
        loop = asyncio.get_event_loop()
        self._results[request_id] = loop.create_future()

    def abort_request(self, request_id: str) -> None:
        req = self.requests.pop(request_id, None)
        if req is None:
            return
        req.status = SchedulerStatus.ABORTED
        for lst in (self.waiting, self.running):
            if req in lst:
                lst.remove(req)
                if lst is self.running:
                    self.resources.free(req)
        fut = self._results.pop(request_id, None)
        if fut is not None and not fut.done():
            fut.cancel()
        q = self._streams.pop(request_id, None)
        if q is not None:
            q.put_nowait(None)

    async def get_result(self, request_id: str) -> Any:
        if request_id in self._finished:
            return self._finished[request_id]
        fut = self._results.get(request_id)
        if fut is None:
            raise KeyError(request_id)
        return await fut

    def stream(self, request_id: str) -> asyncio.Queue:
        q = self._streams.get(request_id)
        if q is None:
            q = self._streams[request_id] = asyncio.Queue()
        return q

    def has_work(self) -> bool:
        return bool(self.waiting or any(r.status == SchedulerStatus.RUNNING for r in self.running))

    def schedule(self) -> SchedulerOutput | None:
        sel = self.planner.select_requests(self.waiting, self.running, self.resources)
        if not sel:
            return None
        for r in sel:
            if r in self.waiting:
                self.waiting.remove(r)
                self.resources.allocate(r)
                self.running.append(r)
            r.status = SchedulerStatus.RUNNING
        self._step += 1
        return SchedulerOutput(sel, self.planner.build_batch(sel), self._step)

    def update(self, sched_out: SchedulerOutput, outputs: dict[str, RequestOutput]) -> None:
        for r in sched_out.requests:
            if r.status != SchedulerStatus.RUNNING:
                continue  # aborted while the step ran (overlap-safe)
            out = outputs.get(r.request_id)
            if out is None:
                continue
            r.num_steps += 1
            self.controller.update_request(r, out.data)
            q = self._streams.get(r.request_id)
            if q is not None:
                q.put_nowait(out.data)
            if out.finished or self.controller.is_finished(r, out.data):
                self._finish_request(r, out.data)

    def fail(self, sched_out: SchedulerOutput, exc: BaseException) -> None:
        for r in sched_out.requests:
            self._finish_request(r, None, exc)

    def _finish_request(self, r: SchedulerRequest, data: Any, exc: BaseException | None = None) -> None:
        r.status = SchedulerStatus.FINISHED
        r.finish_time = time.perf_counter()
        if r in self.running:
            self.running.remove(r)
            self.resources.free(r)
        self.requests.pop(r.request_id, None)
        fut = self._results.pop(r.request_id, None)
        result = r.data if data is None else data
        if fut is not None and not fut.done():
            if exc is not None:
                fut.set_exception(exc)
            else:
                fut.set_result(result)
        if exc is None:
            self._finished[r.request_id] = result
            while len(self._finished) > self.max_retained:
                self._finished.popitem(last=False)
        q = self._streams.pop(r.request_id, None)
        if q is not None:
            q.put_nowait(None)
