"""Runs ``model(**inputs)`` in a worker thread.  Batch mode consumes the whole
payload (after prefetching inbound stream chunks); streaming mode runs one
forward per inbound chunk and pushes each output to the stream target
(sglang_omni/executors/direct_model_executor.py:20-187)."""
from __future__ import annotations

import asyncio
from typing import Any, Callable

import torch

from ..proto import StagePayload
from .interface import Executor, ResultQueueMixin
from .preprocessing_executor import StageError


class DirectModelExecutor(ResultQueueMixin, Executor):
    def __init__(self, model: Callable[..., Any], input_builder: Callable[[StagePayload], dict] | None = None,
                 output_builder: Callable[[StagePayload, Any], Any] | None = None, streaming: bool = False,
                 stream_target: str | None = None):
        super().__init__()
        self.model = model
        self.input_builder = input_builder or (lambda p: p.data if isinstance(p.data, dict) else {"x": p.data})
        self.output_builder = output_builder or (lambda p, out: out)
        self.streaming = streaming
        self.stream_target = stream_target
        self._tasks: dict[str, asyncio.Task] = {}

    def _forward(self, inputs: dict):
        with torch.inference_mode():
            return self.model(**inputs)

    async def add_request(self, payload: StagePayload) -> None:
        rid = payload.request_id

        async def run():
            try:
                if self.streaming and self._mailbox is not None:
                    outs = []
                    while True:
                        item = await self._mailbox.get(rid)
                        if item is None:
                            break
                        out = await asyncio.to_thread(self._forward, self.input_builder(
                            StagePayload(rid, payload.request, item.data)))
                        outs.append(out)
                        if self._stream_fn is not None:
                            self._stream_fn(rid, out, self.stream_target)
                    data = self.output_builder(payload, outs)
                else:
                    out = await asyncio.to_thread(self._forward, self.input_builder(payload))
                    data = self.output_builder(payload, out)
                self._results().put_nowait(StagePayload(rid, payload.request, data))
            except asyncio.CancelledError:
                raise
            except Exception as exc:
                self._results().put_nowait(StageError(rid, f"{type(exc).__name__}: {exc}"))
            finally:
                self._tasks.pop(rid, None)

        self._tasks[rid] = asyncio.ensure_future(run())

    async def abort(self, request_id):
        t = self._tasks.pop(request_id, None)
        if t is not None:
            t.cancel()
