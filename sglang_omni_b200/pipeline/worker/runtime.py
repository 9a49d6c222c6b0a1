"""Stage worker: drives one executor.

Per work item: register the result future before submitting (no lost
completions), bootstrap streaming targets with the input payload, submit to
the executor, forward the executor's client-facing stream to the coordinator,
then route the result with ``get_next``: None = terminal (CompleteMessage to
the coordinator), a stage name or a list of names = fan-out through the data
plane.  Inter-stage streaming goes through a single send loop per worker so
chunk order per request is preserved; ``stream_fn`` is safe to call from any
thread (engine threads call it).  Failures fail only the request they belong
to, and are propagated to its stream targets.

Reference counterpart: sglang_omni/pipeline/worker/runtime.py:42-673.
"""
from __future__ import annotations

import asyncio
import logging
from typing import Any, Callable

from ...proto import CompleteMessage, DataReadyMessage, StagePayload, StreamMessage
from ..control_plane import StageControlPlane
from ..stage.work import WorkDescriptor
from .data_plane import DataPlaneAdapter

log = logging.getLogger(__name__)


class Worker:
    def __init__(self, stage_name: str, executor, get_next: Callable[[str, StagePayload], Any],
                 data_plane: DataPlaneAdapter, control_plane: StageControlPlane, endpoints: dict[str, str],
                 stream_targets: list[tuple[str, bool]] | None = None, stage_id: int | None = None,
                 relay_ranks: dict[str, int] | None = None, stream_finish_timeout: float = 10.0):
        self.stage_name = stage_name
        self.executor = executor
        self.get_next = get_next
        self.data_plane = data_plane
        self.cp = control_plane
        self.endpoints = endpoints
        self.stream_targets = list(stream_targets or [])
        self.stage_id = stage_id
        self.relay_ranks = relay_ranks or {}
        self.stream_finish_timeout = stream_finish_timeout
        self.queue: asyncio.Queue[WorkDescriptor] = asyncio.Queue()
        self._pending: dict[str, asyncio.Future] = {}
        self._tasks: set[asyncio.Task] = set()
        self._loop: asyncio.AbstractEventLoop | None = None
        self._stream_q: asyncio.Queue | None = None
        self._chunk_ids: dict[tuple[str, str], int] = {}
        self._aborted: set[str] = set()

    # ------------------------------------------------------------------ lifecycle
    async def start(self):
        self._loop = asyncio.get_running_loop()
        self._stream_q = asyncio.Queue()
        self.executor.set_stream_fn(self._stream_fn)
        if self.stream_targets and hasattr(self.executor, "set_stream_target"):
            self.executor.set_stream_target([t for t, _ in self.stream_targets])
        await self.executor.start()
        self._spawn(self._dispatch_results())
        self._spawn(self._stream_send_loop())

    async def stop(self):
        for t in list(self._tasks):
            t.cancel()
        await self.executor.stop()

    def _spawn(self, coro):
        t = asyncio.ensure_future(coro)
        self._tasks.add(t)
        t.add_done_callback(self._tasks.discard)
        return t

    async def run(self):
        while True:
            work = await self.queue.get()
            self._spawn(self._process_request(work))

    # ------------------------------------------------------------------ results
    async def _dispatch_results(self):
        while True:
            try:
                res = await self.executor.get_result()
                fut = self._pending.pop(res.request_id, None)
                if fut is not None and not fut.done():
                    fut.set_result(res)
            except asyncio.CancelledError:
                raise
            except Exception as exc:
                rid = getattr(exc, "request_id", None)
                fut = self._pending.pop(rid, None) if rid is not None else None
                if fut is not None and not fut.done():
                    fut.set_exception(exc)
                else:
                    log.exception("executor error without a request id in stage %s", self.stage_name)
                    await asyncio.sleep(0.1)

    # ------------------------------------------------------------------ streaming
    def _stream_fn(self, request_id: str, data: Any, target_stage: str | None = None, metadata: dict | None = None):
        item = (request_id, data, target_stage, metadata or {})
        try:
            running = asyncio.get_running_loop()
        except RuntimeError:
            running = None
        if running is self._loop:
            self._stream_q.put_nowait(item)
        else:
            self._loop.call_soon_threadsafe(self._stream_q.put_nowait, item)

    def _targets_for(self, target_stage: str | None) -> list[str]:
        if target_stage is not None:
            return [target_stage]
        return [t for t, _ in self.stream_targets]

    async def _stream_send_loop(self):
        while True:
            rid, data, target, meta = await self._stream_q.get()
            if rid in self._aborted:
                continue
            for t in self._targets_for(target):
                try:
                    if meta.get("_signal") == "done":
                        msg = DataReadyMessage(rid, self.stage_name, t, None, chunk_id=-1, is_done=True)
                    elif meta.get("_signal") == "error":
                        msg = DataReadyMessage(rid, self.stage_name, t, None, chunk_id=-1, error=meta["error"])
                    else:
                        key = (rid, t)
                        cid = self._chunk_ids.get(key, 0)
                        self._chunk_ids[key] = cid + 1
                        md = await self.data_plane.write_blob(rid, {"data": data, "metadata": meta},
                                                              dst=self.relay_ranks.get(t))
                        msg = DataReadyMessage(rid, self.stage_name, t, md, chunk_id=cid)
                    await self.cp.send_to_stage(self.endpoints[t], msg)
                except Exception:
                    log.exception("stream send %s -> %s failed for %s", self.stage_name, t, rid)

    async def _finish_streams(self, rid: str, error: str | None = None):
        targets = [t for t, _ in self.stream_targets]
        if not targets:
            return
        sig = {"_signal": "error", "error": error} if error else {"_signal": "done"}
        self._stream_q.put_nowait((rid, None, None, sig))
        for t in targets:
            self._chunk_ids.pop((rid, t), None)

    async def _forward_client_stream(self, rid: str, it):
        try:
            seq = 0
            async for chunk in it:
                modality = chunk.get("modality") if isinstance(chunk, dict) else None
                await self.cp.send_to_coordinator(StreamMessage(rid, self.stage_name, chunk, self.stage_id,
                                                                self.stage_name, modality, seq))
                seq += 1
        except asyncio.CancelledError:
            raise
        except Exception:
            log.exception("client stream of %s failed in %s", rid, self.stage_name)

    # ------------------------------------------------------------------ routing
    async def _send_payload(self, target: str, payload: StagePayload):
        md = await self.data_plane.write_payload(payload.request_id, payload, dst=self.relay_ranks.get(target))
        await self.cp.send_to_stage(self.endpoints[target],
                                    DataReadyMessage(payload.request_id, self.stage_name, target, md))

    async def _process_request(self, work: WorkDescriptor):
        rid = work.request_id
        fut = self._loop.create_future()
        self._pending[rid] = fut  # registered before add_request: no lost completion
        stream_task = None
        try:
            for target, bootstrap in self.stream_targets:
                if bootstrap:
                    await self._send_payload(target, work.payload)
            await self.executor.add_request(work.payload)
            it = self.executor.stream(rid)
            if it is not None:
                stream_task = self._spawn(self._forward_client_stream(rid, it))
            result = await fut
        except asyncio.CancelledError:
            self._pending.pop(rid, None)
            raise
        except Exception as exc:
            self._pending.pop(rid, None)
            err = f"{self.stage_name}: {exc}"
            await self._finish_streams(rid, error=err)
            if rid not in self._aborted:
                await self.cp.send_to_coordinator(CompleteMessage(rid, self.stage_name, False, None, err))
            return
        if stream_task is not None:
            try:
                await asyncio.wait_for(asyncio.shield(stream_task), self.stream_finish_timeout)
            except asyncio.TimeoutError:
                log.warning("client stream of %s did not finish in %.1fs", rid, self.stream_finish_timeout)
        await self._finish_streams(rid)
        if rid in self._aborted:
            return
        try:
            nxt = self.get_next(rid, result)
        except Exception as exc:
            await self.cp.send_to_coordinator(CompleteMessage(rid, self.stage_name, False, None,
                                                              f"{self.stage_name}.get_next: {exc}"))
            return
        if nxt is None:
            await self.cp.send_to_coordinator(CompleteMessage(rid, self.stage_name, True, result.data))
            return
        for t in ([nxt] if isinstance(nxt, str) else list(nxt)):
            await self._send_payload(t, result)

    async def abort(self, rid: str):
        self._aborted.add(rid)
        if len(self._aborted) > 10000:
            self._aborted.pop()
        fut = self._pending.pop(rid, None)
        if fut is not None and not fut.done():
            fut.cancel()
        await self.executor.abort(rid)
