"""Chains the executors of fused (co-located, adjacent) stages inside one
worker: intermediate steps run one request at a time under a lock, the last
executor runs concurrently and owns streaming
(sglang_omni/executors/fused_executor.py:15-96)."""
from __future__ import annotations

import asyncio

from ..proto import StagePayload
from .interface import Executor, ResultQueueMixin
from .preprocessing_executor import StageError


class FusedExecutor(ResultQueueMixin, Executor):
    def __init__(self, executors: list[Executor], names: list[str] | None = None):
        super().__init__()
        if not executors:
            raise ValueError("FusedExecutor needs at least one executor")
        self.executors = executors
        self.names = names or [f"step{i}" for i in range(len(executors))]
        self._lock = asyncio.Lock()
        self._pump: asyncio.Task | None = None

    async def start(self):
        for e in self.executors:
            await e.start()

    async def stop(self):
        for e in self.executors:
            await e.stop()
        if self._pump is not None:
            self._pump.cancel()

    def set_stream_fn(self, fn):
        self.executors[-1].set_stream_fn(fn)

    def set_feedback_mailbox(self, mailbox):
        for e in self.executors:
            e.set_feedback_mailbox(mailbox)

    async def _run_intermediate(self, payload: StagePayload) -> StagePayload:
        for e in self.executors[:-1]:
            async with self._lock:
                await e.add_request(payload)
                payload = await e.get_result()
        return payload

    async def add_request(self, payload: StagePayload) -> None:
        if self._pump is None:
            self._pump = asyncio.ensure_future(self._forward_results())

        async def run():
            try:
                p = await self._run_intermediate(payload)
                await self.executors[-1].add_request(p)
            except Exception as exc:
                rid = getattr(exc, "request_id", payload.request_id)
                self._results().put_nowait(StageError(rid, str(exc)))

        asyncio.ensure_future(run())

    async def _forward_results(self):
        last = self.executors[-1]
        while True:
            try:
                self._results().put_nowait(await last.get_result())
            except asyncio.CancelledError:
                raise
            except Exception as exc:
                self._results().put_nowait(exc)

    def stream(self, request_id):
        return self.executors[-1].stream(request_id)

    async def abort(self, request_id):
        for e in self.executors:
            await e.abort(request_id)


def create_fused_executor(executors: list[Executor], names: list[str] | None = None) -> FusedExecutor:
    return FusedExecutor(executors, names)
