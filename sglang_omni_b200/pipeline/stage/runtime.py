"""Stage runtime: receives submits, data-ready hand-offs, stream chunks,
aborts and profiler commands; feeds its workers.

* Full payloads are read from the relay as soon as they arrive (releasing the
  sender's credit) and go through the input handler (direct or aggregated
  fan-in) and the sticky router to a worker.
* Stream chunks (DataReadyMessage with chunk_id) land in the stage's
  StreamQueue, which executors read as their inbound mailbox; chunks that
  arrive before the request reaches a worker are kept.
* Aborts (PUB/SUB) clean up router affinity, pending fan-in, stream queue,
  relay buffers and every worker's executor state.

Reference counterpart: sglang_omni/pipeline/stage/runtime.py:43-602.
"""
from __future__ import annotations

import asyncio
import logging
import os

from ...proto import (AbortMessage, CompleteMessage, DataReadyMessage, ProfilerStartMessage, ProfilerStopMessage,
                      ShutdownMessage, StageStatsMessage, SubmitMessage)
from ..control_plane import StageControlPlane
from ..worker.data_plane import DataPlaneAdapter
from .input import DirectInput, InputHandler
from .router import WorkerRouter
from .stream_queue import StreamItem, StreamQueue
from .work import WorkDescriptor

log = logging.getLogger(__name__)


class Stage:
    def __init__(self, name: str, control_plane: StageControlPlane, data_plane: DataPlaneAdapter,
                 input_handler: InputHandler | None = None, stream_queue: StreamQueue | None = None):
        self.name = name
        self.cp = control_plane
        self.data_plane = data_plane
        self.input_handler = input_handler or DirectInput()
        self.stream_queue = stream_queue
        self.workers = []
        self.router: WorkerRouter | None = None
        self._running = False
        self._tasks: list[asyncio.Task] = []
        self._profiler = None
        self.messages_received = 0
        # seconds between load reports to the coordinator (0: none)
        self.stats_interval_s = float(os.environ.get("OMNI_STAGE_STATS_S", "1.0"))

    def add_worker(self, worker) -> None:
        self.workers.append(worker)
        if self.stream_queue is not None:
            worker.executor.set_feedback_mailbox(self.stream_queue)
        self.router = WorkerRouter(len(self.workers))

    async def start(self):
        self.cp.start()
        for w in self.workers:
            await w.start()
        self._running = True

    async def stop(self):
        self._running = False
        for t in self._tasks:
            t.cancel()
        for w in self.workers:
            await w.stop()
        self.cp.close()
        self.data_plane.relay.close()

    async def run(self):
        self._tasks = [asyncio.ensure_future(w.run()) for w in self.workers]
        self._tasks.append(asyncio.ensure_future(self._abort_loop()))
        if self.stats_interval_s > 0:
            self._tasks.append(asyncio.ensure_future(self._stats_loop()))
        try:
            while self._running:
                msg = await self.cp.recv()
                self.messages_received += 1
                if isinstance(msg, ShutdownMessage):
                    break
                try:
                    await self._handle_message(msg)
                except Exception as exc:
                    log.exception("stage %s failed to handle %s", self.name, type(msg).__name__)
                    rid = getattr(msg, "request_id", None)
                    if rid is not None:  # fail only this request (fail-fast at the coordinator)
                        try:
                            await self.cp.send_to_coordinator(CompleteMessage(
                                rid, self.name, False, None, f"{self.name}: {type(exc).__name__}: {exc}"))
                        except Exception:
                            log.exception("could not report the failure of %s", rid)
        finally:
            for t in self._tasks:
                t.cancel()

    async def _handle_message(self, msg):
        if isinstance(msg, SubmitMessage):
            self._route(msg.request_id, None, msg.data)
        elif isinstance(msg, DataReadyMessage):
            if msg.chunk_id is None and not msg.is_done and msg.error is None:
                payload = await self.data_plane.read_payload(msg.shm_metadata)
                self._route(msg.request_id, msg.from_stage, payload)
            else:
                await self._handle_stream_chunk(msg)
        elif isinstance(msg, AbortMessage):
            await self._on_abort(msg.request_id)
        elif isinstance(msg, ProfilerStartMessage):
            self._profiler_start(msg)
        elif isinstance(msg, ProfilerStopMessage):
            self._profiler_stop(msg)

    async def _handle_stream_chunk(self, msg: DataReadyMessage):
        if self.stream_queue is None:
            log.warning("stage %s got a stream chunk but has no stream queue", self.name)
            return
        rid = msg.request_id
        if msg.error is not None:
            self.stream_queue.put_error(rid, msg.error, msg.from_stage)
        elif msg.is_done:
            self.stream_queue.put_done(rid, msg.from_stage)
        else:
            blob = await self.data_plane.read_blob(msg.shm_metadata)
            self.stream_queue.put(rid, StreamItem(msg.chunk_id, blob.get("data"), msg.from_stage,
                                                  blob.get("metadata") or {}))

    def _route(self, rid: str, from_stage: str | None, payload):
        ready = self.input_handler.receive(rid, from_stage, payload)
        if ready is None:
            return
        w = self.router.route(rid)
        self.workers[w].queue.put_nowait(WorkDescriptor(rid, ready, from_stage))

    async def _abort_loop(self):
        while True:
            msg = await self.cp.recv_abort()
            if isinstance(msg, AbortMessage):
                await self._on_abort(msg.request_id)

    async def _on_abort(self, rid: str):
        self.input_handler.cancel(rid)
        if self.router is not None:
            self.router.release(rid)
        if self.stream_queue is not None:
            self.stream_queue.close(rid)
        self.data_plane.relay.cleanup(rid)
        for w in self.workers:
            await w.abort(rid)

    # ------------------------------------------------------------------ profiler
    def _profiler_start(self, msg: ProfilerStartMessage):
        from ...profiler.torch_profiler import TorchProfiler

        path = msg.trace_path_template.format(run_id=msg.run_id, stage=self.name)
        self._profiler = TorchProfiler(path + f"_pid{os.getpid()}")
        self._profiler.start()

    def _profiler_stop(self, msg: ProfilerStopMessage):
        if self._profiler is not None:
            self._profiler.stop()
            self._profiler = None

    def stats(self) -> dict:
        """Queue depth over the workers, messages received, and what the executors report
        (an engine's running / waiting requests, KV-cache pages in use)."""
        out = {"queue_depth": sum(w.queue.qsize() for w in self.workers if hasattr(w, "queue")),
               "messages": self.messages_received}
        for w in self.workers:
            fn = getattr(w.executor, "stats", None)
            if fn is None:
                continue
            try:
                for k, v in (fn() or {}).items():
                    if isinstance(v, (int, float)) and not isinstance(v, bool):
                        out[k] = out.get(k, 0) + v
            except Exception:
                log.debug("stats of %s failed", self.name, exc_info=True)
        return out

    async def _stats_loop(self):
        while self._running:
            await asyncio.sleep(self.stats_interval_s)
            try:
                await self.cp.send_to_coordinator(StageStatsMessage(self.name, self.stats()))
            except Exception:
                log.debug("stats report of %s failed", self.name, exc_info=True)

    def health(self) -> dict:
        return {"stage": self.name, "running": self._running, "workers": len(self.workers),
                "messages": self.messages_received, "relay": self.data_plane.relay.health()}
