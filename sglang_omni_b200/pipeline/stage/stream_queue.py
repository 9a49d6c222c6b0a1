"""Per-request streaming queues between stages.

Semantics (sglang_omni/pipeline/stage/stream_queue.py:14-128): chunks are
delivered in order; ``put_done`` / ``put_error`` terminate a stream; puts for
a request that was closed (finished or aborted) are dropped silently; chunks
that arrive before the consumer opened the queue are kept (bounded by
``max_pending`` requests).
"""
from __future__ import annotations

import asyncio
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any


@dataclass
class StreamItem:
    chunk_id: int
    data: Any
    from_stage: str | None = None
    metadata: dict = field(default_factory=dict)


@dataclass
class StreamSignal:
    is_done: bool = False
    error: str | None = None
    from_stage: str | None = None


class StreamQueue:
    def __init__(self, max_pending: int = 4096):
        self.max_pending = max_pending
        self._queues: dict[str, asyncio.Queue] = {}
        self._closed: OrderedDict[str, None] = OrderedDict()

    def open(self, request_id: str) -> asyncio.Queue:
        q = self._queues.get(request_id)
        if q is None:
            q = self._queues[request_id] = asyncio.Queue()
        self._closed.pop(request_id, None)
        return q

    def has(self, request_id: str) -> bool:
        return request_id in self._queues

    def _q(self, request_id: str) -> asyncio.Queue | None:
        if request_id in self._closed:
            return None
        q = self._queues.get(request_id)
        if q is None:
            if len(self._queues) >= self.max_pending:
                return None
            q = self._queues[request_id] = asyncio.Queue()
        return q

    def put(self, request_id: str, item: StreamItem) -> bool:
        q = self._q(request_id)
        if q is None:
            return False
        q.put_nowait(item)
        return True

    def put_done(self, request_id: str, from_stage: str | None = None) -> None:
        q = self._q(request_id)
        if q is not None:
            q.put_nowait(StreamSignal(is_done=True, from_stage=from_stage))

    def put_error(self, request_id: str, error: str, from_stage: str | None = None) -> None:
        q = self._q(request_id)
        if q is not None:
            q.put_nowait(StreamSignal(error=error, from_stage=from_stage))

    async def get(self, request_id: str, timeout: float | None = None) -> StreamItem | None:
        """Next chunk; None at end of stream; raises RuntimeError on a stream error."""
        item, _ = await self.get_with_source(request_id, timeout)
        return item

    async def get_with_source(self, request_id: str, timeout: float | None = None):
        q = self.open(request_id)
        if timeout is None:
            item = await q.get()
        else:
            item = await asyncio.wait_for(q.get(), timeout)
        if isinstance(item, StreamSignal):
            if item.error is not None:
                raise RuntimeError(f"stream error from {item.from_stage}: {item.error}")
            return None, item.from_stage
        return item, item.from_stage

    def get_nowait(self, request_id: str):
        q = self._queues.get(request_id)
        if q is None or q.empty():
            return None
        return q.get_nowait()

    def close(self, request_id: str) -> None:
        self._queues.pop(request_id, None)
        self._closed[request_id] = None
        while len(self._closed) > 10000:
            self._closed.popitem(last=False)
