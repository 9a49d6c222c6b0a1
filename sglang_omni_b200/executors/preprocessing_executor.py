"""Runs a sync (in a worker thread) or async preprocessing function per request
(sglang_omni/executors/preprocessing_executor.py:15-58)."""
from __future__ import annotations

import asyncio
import inspect

from ..proto import StagePayload
from .interface import Executor, ResultQueueMixin


class StageError(RuntimeError):
    """An executor failed one request; carries its id so only that request fails."""

    def __init__(self, request_id: str, message: str):
        super().__init__(message)
        self.request_id = request_id


class PreprocessingExecutor(ResultQueueMixin, Executor):
    def __init__(self, fn):
        super().__init__()
        self.fn = fn
        self._tasks: dict[str, asyncio.Task] = {}

    async def add_request(self, payload: StagePayload) -> None:
        async def run():
            try:
                if inspect.iscoroutinefunction(self.fn):
                    out = await self.fn(payload)
                else:
                    out = await asyncio.to_thread(self.fn, payload)
                if not isinstance(out, StagePayload):
                    out = StagePayload(payload.request_id, payload.request, out)
                self._results().put_nowait(out)
            except asyncio.CancelledError:
                raise
            except Exception as exc:
                self._results().put_nowait(StageError(payload.request_id, f"{type(exc).__name__}: {exc}"))
            finally:
                self._tasks.pop(payload.request_id, None)

        self._tasks[payload.request_id] = asyncio.ensure_future(run())

    async def abort(self, request_id: str) -> None:
        t = self._tasks.pop(request_id, None)
        if t is not None:
            t.cancel()
