"""Engine contract (sglang_omni/engines/base.py:11-44) and the one-forward-per-
request module engine (sglang_omni/engines/async_module.py:15)."""
from __future__ import annotations

import abc
import asyncio
from typing import Any, Callable

import torch


class Engine(abc.ABC):
    @abc.abstractmethod
    async def add_request(self, request_id: str, data: Any) -> None: ...

    @abc.abstractmethod
    async def get_result(self, request_id: str) -> Any: ...

    async def abort(self, request_id: str) -> None:
        pass

    def transform_output(self, output: Any) -> Any:
        return output

    async def generate(self, request_id: str, data: Any, on_chunk=None, stream_fn=None) -> Any:
        await self.add_request(request_id, data)
        return await self.get_result(request_id)


class AsyncModuleEngine(Engine):
    """Runs ``module(**data)`` (or ``module(data)``) per request in a worker thread."""

    def __init__(self, module: Callable[..., Any]):
        self.module = module
        self._futs: dict[str, asyncio.Future] = {}

    def _run(self, data):
        with torch.inference_mode():
            return self.module(**data) if isinstance(data, dict) else self.module(data)

    async def add_request(self, request_id, data):
        self._futs[request_id] = asyncio.ensure_future(asyncio.to_thread(self._run, data))

    async def get_result(self, request_id):
        return self.transform_output(await self._futs.pop(request_id))

    async def abort(self, request_id):
        f = self._futs.pop(request_id, None)
        if f is not None:
            f.cancel()
