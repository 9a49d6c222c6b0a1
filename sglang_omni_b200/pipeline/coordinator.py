"""Coordinator: request registry, submission to the entry stage, completion
loop, per-request stream queues, multi-terminal fan-in, fail-fast, abort.

Lifecycle PENDING -> RUNNING -> COMPLETED / FAILED / ABORTED.  With several
terminal stages (e.g. text ``decode`` and audio ``code2wav``) the request
completes when every terminal reported, and the result is {stage: result}.
Any stage failure fails the request at once and broadcasts an abort so the
other stages drop its state.

Reference counterpart: sglang_omni/pipeline/coordinator.py:24-394.
"""
from __future__ import annotations

import asyncio
import logging
import time
from dataclasses import dataclass, field
from typing import Any, AsyncIterator

from ..proto import (AbortMessage, CompleteMessage, OmniRequest, ProfilerStartMessage, ProfilerStopMessage,
                     RequestInfo, RequestState, ShutdownMessage, StagePayload, StageStatsMessage, StreamMessage,
                     SubmitMessage)
from .control_plane import CoordinatorControlPlane

log = logging.getLogger(__name__)


@dataclass
class _Req:
    info: RequestInfo
    future: asyncio.Future
    stream: asyncio.Queue | None = None
    terminal_results: dict[str, Any] = field(default_factory=dict)
    submitted_at: float = field(default_factory=time.perf_counter)
    last_seq: dict[str, int] = field(default_factory=dict)   # stage -> last stream chunk number seen


class Coordinator:
    def __init__(self, completion_endpoint: str, abort_endpoint: str, entry_stage: str,
                 terminal_stages: list[str] | None = None, max_retained: int = 10000,
                 request_timeout_s: float | None = None):
        """``request_timeout_s``: a request that has not completed this long after its
        submission fails with a TimeoutError and is aborted in every stage (a lost
        completion or a stalled stage then ends in an error instead of a hang)."""
        self.request_timeout_s = request_timeout_s
        self._watchdog: asyncio.Task | None = None
        self.cp = CoordinatorControlPlane(completion_endpoint, abort_endpoint)
        self.entry_stage = entry_stage
        self.terminal_stages = list(terminal_stages or [])
        self.stage_endpoints: dict[str, str] = {}
        self.stage_stats: dict[str, dict] = {}    # last load report of each stage
        self._reqs: dict[str, _Req] = {}
        self._done_states: dict[str, RequestState] = {}
        self.max_retained = max_retained
        self._loop_task: asyncio.Task | None = None
        self.running = False

    def register_stage(self, name: str, endpoint: str) -> None:
        self.stage_endpoints[name] = endpoint

    async def start(self):
        await self.cp.start()
        self.running = True
        if self.request_timeout_s:
            self._watchdog = asyncio.ensure_future(self._deadline_loop())

    async def _deadline_loop(self):
        period = max(0.01, min(1.0, self.request_timeout_s / 4))
        while True:
            await asyncio.sleep(period)
            now = time.perf_counter()
            late = [rid for rid, r in self._reqs.items() if now - r.submitted_at > self.request_timeout_s]
            for rid in late:
                log.warning("request %s exceeded its %.1fs deadline", rid, self.request_timeout_s)
                try:
                    await self.cp.broadcast(AbortMessage(rid))
                except Exception:
                    log.exception("abort broadcast for %s failed", rid)
                self._finish(rid, RequestState.FAILED,
                             exc=TimeoutError(f"request {rid} did not complete within {self.request_timeout_s}s"))

    async def stop(self):
        self.running = False
        for ep in self.stage_endpoints.values():
            try:
                await self.cp.send_to_stage(ep, ShutdownMessage())
            except Exception:
                pass
        if self._loop_task is not None:
            self._loop_task.cancel()
        if self._watchdog is not None:
            self._watchdog.cancel()
        self.cp.close()

    # ------------------------------------------------------------------ submission
    async def _submit_request(self, request_id: str, request: OmniRequest, stream: bool) -> _Req:
        if request_id in self._reqs:
            raise ValueError(f"duplicate request id {request_id}")
        loop = asyncio.get_running_loop()
        r = _Req(RequestInfo(request_id, RequestState.RUNNING, self.entry_stage), loop.create_future(),
                 asyncio.Queue() if stream else None)
        self._reqs[request_id] = r
        payload = StagePayload(request_id=request_id, request=request, data=request.inputs)
        await self.cp.send_to_stage(self.stage_endpoints[self.entry_stage], SubmitMessage(request_id, payload))
        return r

    async def submit(self, request_id: str, request: OmniRequest) -> Any:
        r = await self._submit_request(request_id, request, stream=False)
        return await r.future

    async def stream(self, request_id: str, request: OmniRequest) -> AsyncIterator[Any]:
        """Yields StreamMessage chunks, then a final CompleteMessage-like dict."""
        r = await self._submit_request(request_id, request, stream=True)
        while True:
            get = asyncio.ensure_future(r.stream.get())
            done, _ = await asyncio.wait({get, r.future}, return_when=asyncio.FIRST_COMPLETED)
            if get in done:
                yield get.result()
                continue
            get.cancel()
            while not r.stream.empty():  # drain chunks that raced the completion
                yield r.stream.get_nowait()
            yield {"type": "complete", "result": r.future.result()}  # raises on failure
            return

    async def abort(self, request_id: str) -> bool:
        r = self._reqs.get(request_id)
        if r is None:
            return False
        await self.cp.broadcast(AbortMessage(request_id))
        self._finish(request_id, RequestState.ABORTED, exc=asyncio.CancelledError(f"request {request_id} aborted"))
        return True

    # ------------------------------------------------------------------ completion loop
    async def run_completion_loop(self):
        while True:
            msg = await self.cp.recv()
            try:
                if isinstance(msg, CompleteMessage):
                    await self._handle_completion(msg)
                elif isinstance(msg, StageStatsMessage):
                    self.stage_stats[msg.stage] = {**msg.stats, "_t": time.monotonic()}
                elif isinstance(msg, StreamMessage):
                    r = self._reqs.get(msg.request_id)
                    if r is not None and r.stream is not None:
                        if msg.seq is not None:   # a duplicated (re-sent) chunk is dropped
                            if msg.seq <= r.last_seq.get(msg.from_stage, -1):
                                continue
                            r.last_seq[msg.from_stage] = msg.seq
                        r.stream.put_nowait(msg)
            except Exception:
                log.exception("coordinator failed on %s", type(msg).__name__)

    def start_completion_loop(self):
        self._loop_task = asyncio.ensure_future(self.run_completion_loop())
        return self._loop_task

    async def _handle_completion(self, msg: CompleteMessage):
        r = self._reqs.get(msg.request_id)
        if r is None:
            return
        if not msg.success:
            await self.cp.broadcast(AbortMessage(msg.request_id))
            r.info.error = msg.error
            self._finish(msg.request_id, RequestState.FAILED, exc=RuntimeError(msg.error or "stage failed"))
            return
        terminals = self.terminal_stages or [msg.from_stage]
        r.terminal_results[msg.from_stage] = msg.result
        if all(t in r.terminal_results for t in terminals):
            result = r.terminal_results[terminals[0]] if len(terminals) == 1 else dict(r.terminal_results)
            r.info.result = result
            self._finish(msg.request_id, RequestState.COMPLETED, result=result)

    def _finish(self, rid: str, state: RequestState, result: Any = None, exc: BaseException | None = None):
        r = self._reqs.pop(rid, None)
        if r is None:
            return
        r.info.state = state
        if not r.future.done():
            if exc is not None:
                r.future.set_exception(exc)
            else:
                r.future.set_result(result)
        self._done_states[rid] = state
        while len(self._done_states) > self.max_retained:
            self._done_states.pop(next(iter(self._done_states)))

    # ------------------------------------------------------------------ profiler / health
    async def start_profile(self, run_id: str, trace_path_template: str):
        for ep in self.stage_endpoints.values():
            await self.cp.send_to_stage(ep, ProfilerStartMessage(run_id, trace_path_template))

    async def stop_profile(self, run_id: str):
        for ep in self.stage_endpoints.values():
            await self.cp.send_to_stage(ep, ProfilerStopMessage(run_id))

    def health(self) -> dict:
        counts = {s.value: 0 for s in RequestState}
        counts[RequestState.RUNNING.value] = len(self._reqs)
        for st in self._done_states.values():
            counts[st.value] += 1
        return {"running": self.running, "requests": counts, "stages": list(self.stage_endpoints),
                "stage_stats": self.latest_stage_stats()}

    def latest_stage_stats(self) -> dict:
        """Each stage's last load report, with its age in seconds."""
        now = time.monotonic()
        return {n: {**{k: v for k, v in st.items() if k != "_t"}, "age_s": round(now - st["_t"], 3)}
                for n, st in self.stage_stats.items()}
