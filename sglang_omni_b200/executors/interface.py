"""Executor contract between a stage worker and whatever computes the stage
(sglang_omni/executors/interface.py:11-42): add_request(payload), get_result()
in completion order, abort(request_id), optional per-request ``stream``, and
hooks for inter-stage streaming (``set_stream_fn``) and inbound chunks /
feedback (``set_feedback_mailbox``)."""
from __future__ import annotations

import abc
import asyncio
from typing import Any, AsyncIterator, Callable

from ..proto import StagePayload

# stream_fn(request_id, data, target_stage=None, metadata=None) -> None
StreamFn = Callable[..., Any]


class Executor(abc.ABC):
    def __init__(self):
        self._stream_fn: StreamFn | None = None
        self._mailbox = None

    async def start(self) -> None:
        pass

    async def stop(self) -> None:
        pass

    @abc.abstractmethod
    async def add_request(self, payload: StagePayload) -> None: ...

    @abc.abstractmethod
    async def get_result(self) -> StagePayload: ...

    async def abort(self, request_id: str) -> None:
        pass

    def stream(self, request_id: str) -> AsyncIterator[Any] | None:
        """Async iterator of client-facing stream chunks for this request, or None."""
        return None

    def set_stream_fn(self, fn: StreamFn | None) -> None:
        self._stream_fn = fn

    def set_feedback_mailbox(self, mailbox) -> None:
        self._mailbox = mailbox

    def set_stream_target(self, targets: list[str]) -> None:
        self._stream_targets = list(targets)


class ResultQueueMixin:
    """Completion-order result delivery shared by the concrete executors."""

    def _init_results(self):
        self._result_q: asyncio.Queue | None = None

    def _results(self) -> asyncio.Queue:
        if getattr(self, "_result_q", None) is None:
            self._result_q = asyncio.Queue()
        return self._result_q

    async def get_result(self) -> StagePayload:
        item = await self._results().get()
        if isinstance(item, BaseException):
            raise item
        return item
