"""Adapts an Engine (add_request / get_result / stream / abort) to the executor
contract: builds the engine request from the payload (optionally after
prefetching every inbound stream chunk), turns the engine output back into a
payload, forwards per-token stream chunks, and records ``engine_time_s``
(sglang_omni/executors/engine_executor.py:16-179)."""
from __future__ import annotations

import asyncio
import time
from typing import Any, Callable

from ..proto import StagePayload
from .interface import Executor, ResultQueueMixin
from .preprocessing_executor import StageError


class EngineExecutor(ResultQueueMixin, Executor):
    def __init__(self, engine, request_builder: Callable[[StagePayload], Any],
                 result_builder: Callable[[StagePayload, Any], StagePayload] | None = None,
                 stream_builder: Callable[[StagePayload, Any], Any] | None = None,
                 prefetch_stream: bool = False):
        super().__init__()
        self.engine = engine
        self.request_builder = request_builder
        self.result_builder = result_builder
        self.stream_builder = stream_builder
        self.prefetch_stream = prefetch_stream
        self._tasks: dict[str, asyncio.Task] = {}
        self._streams: dict[str, asyncio.Queue] = {}


    def stats(self) -> dict:
        """Requests in this executor, plus the engine's own counters when it reports any."""
        out = {"requests_active": len(self._tasks)}
        fn = getattr(self.engine, "stats", None)
        if fn is not None:
            out.update(fn())
        return out
    async def start(self):
        if hasattr(self.engine, "start"):
            r = self.engine.start()
            if asyncio.iscoroutine(r):
                await r

    async def stop(self):
        if hasattr(self.engine, "stop"):
            r = self.engine.stop()
            if asyncio.iscoroutine(r):
                await r

    async def _prefetch(self, payload: StagePayload):
        chunks = []
        if self._mailbox is None:
            return chunks
        while True:
            item = await self._mailbox.get(payload.request_id)
            if item is None:
                break
            chunks.append(item.data)
        return chunks

    async def add_request(self, payload: StagePayload) -> None:
        rid = payload.request_id
        if self.stream_builder is not None:
            self._streams[rid] = asyncio.Queue()

        async def run():
            t0 = time.perf_counter()
            try:
                if self.prefetch_stream:
                    payload.data = {"payload": payload.data, "stream_chunks": await self._prefetch(payload)}
                req = self.request_builder(payload)
                if asyncio.iscoroutine(req):
                    req = await req
                sq = self._streams.get(rid)

                def on_chunk(chunk):
                    if sq is not None and self.stream_builder is not None:
                        out = self.stream_builder(payload, chunk)
                        if out is not None:
                            sq.put_nowait(out)

                out = await self.engine.generate(rid, req, on_chunk=on_chunk, stream_fn=self._stream_fn)
                res = self.result_builder(payload, out) if self.result_builder else StagePayload(rid, payload.request, out)
                meta = res.request.metadata
                meta["engine_time_s"] = meta.get("engine_time_s", 0.0) + (time.perf_counter() - t0)
                self._results().put_nowait(res)
            except asyncio.CancelledError:
                raise
            except Exception as exc:
                self._results().put_nowait(StageError(rid, f"{type(exc).__name__}: {exc}"))
            finally:
                sq = self._streams.get(rid)
                if sq is not None:
                    sq.put_nowait(None)
                self._tasks.pop(rid, None)

        self._tasks[rid] = asyncio.ensure_future(run())

    def stream(self, request_id: str):
        q = self._streams.get(request_id)
        if q is None:
            return None

        async def gen():
            try:
                while True:
                    item = await q.get()
                    if item is None:
                        return
                    yield item
            finally:
                self._streams.pop(request_id, None)

        return gen()

    async def abort(self, request_id: str) -> None:
        if hasattr(self.engine, "abort"):
            r = self.engine.abort(request_id)
            if asyncio.iscoroutine(r):
                await r
        t = self._tasks.pop(request_id, None)
        if t is not None:
            t.cancel()
        q = self._streams.pop(request_id, None)
        if q is not None:
            q.put_nowait(None)
