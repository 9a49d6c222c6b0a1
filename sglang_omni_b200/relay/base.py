"""Relay: moves tensor payloads between stages; the control message carries
only the relay metadata.

Contract (sglang_omni/relay/base.py:14-158): ``put_async(buffer, request_id)``
returns a RelayOperation whose ``metadata`` the receiver passes to
``get_async(metadata)``; ``wait_for_completion(timeout)`` bounds every wait
(30 s default); ``@register_relay`` / ``create_relay(type, **kw)`` build relays
by name, passing only the kwargs the constructor accepts; ``CreditAllocator``
bounds the number of in-flight transfers per relay.
"""
from __future__ import annotations

import abc
import asyncio
import inspect
from typing import Any

import torch

RELAY_REGISTRY: dict[str, type] = {}


def register_relay(name: str):
    def deco(cls):
        RELAY_REGISTRY[name] = cls
        cls.relay_type = name
        return cls

    return deco


def create_relay(relay_type: str, **kwargs) -> "Relay":
    cls = RELAY_REGISTRY.get(relay_type)
    if cls is None:
        # import lazily so optional backends register themselves
        from . import inproc, ipc, nccl, shm  # noqa: F401
        cls = RELAY_REGISTRY.get(relay_type)
    if cls is None:
        raise ValueError(f"unknown relay type {relay_type!r}; known: {sorted(RELAY_REGISTRY)}")
    params = inspect.signature(cls.__init__).parameters
    if any(p.kind == p.VAR_KEYWORD for p in params.values()):
        return cls(**kwargs)
    return cls(**{k: v for k, v in kwargs.items() if k in params})


class RelayOperation:
    def __init__(self, metadata: dict[str, Any] | None = None, future: asyncio.Future | None = None,
                 result: Any = None):
        self.metadata = metadata or {}
        self._future = future
        self.result = result

    async def wait_for_completion(self, timeout: float = 30.0) -> Any:
        if self._future is None:
            return self.result
        self.result = await asyncio.wait_for(self._future, timeout)
        return self.result


class Relay(abc.ABC):
    relay_type = "base"

    @abc.abstractmethod
    async def put_async(self, buffer: torch.Tensor, request_id: str) -> RelayOperation: ...

    @abc.abstractmethod
    async def get_async(self, metadata: dict[str, Any], dest: torch.Tensor | None = None) -> RelayOperation:
        """The operation's result is the received buffer."""

    def cleanup(self, request_id: str) -> None:
        pass

    def close(self) -> None:
        pass

    def health(self) -> dict[str, Any]:
        return {"type": self.relay_type, "ok": True}


class CreditAllocator:
    """asyncio pool of transfer credits (slot ids)."""

    def __init__(self, credits: int):
        self.credits = max(1, credits)
        self._q: asyncio.Queue | None = None

    def _queue(self) -> asyncio.Queue:
        if self._q is None:
            self._q = asyncio.Queue()
            for i in range(self.credits):
                self._q.put_nowait(i)
        return self._q

    async def acquire(self, timeout: float = 30.0) -> int:
        return await asyncio.wait_for(self._queue().get(), timeout)

    def release(self, slot: int) -> None:
        self._queue().put_nowait(slot)

    @property
    def available(self) -> int:
        return self._queue().qsize()
