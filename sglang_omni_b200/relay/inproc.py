"""Same-process relay: hands the tensor object itself to the receiving stage
(zero copy, device tensors stay where they are).  Used when every stage runs
in one process (the single-process pipeline runner)."""
from __future__ import annotations

import itertools
import threading

import torch

from .base import Relay, RelayOperation, register_relay

_OBJECTS: dict[int, torch.Tensor] = {}
_LOCK = threading.Lock()
_IDS = itertools.count(1)


@register_relay("inproc")
class InprocRelay(Relay):
    def __init__(self, device: str = "cpu", **_):
        self.device = device
        self._by_request: dict[str, list[int]] = {}

    async def put_async(self, buffer, request_id):
        h = next(_IDS)
        with _LOCK:
            _OBJECTS[h] = buffer
        self._by_request.setdefault(request_id, []).append(h)
        return RelayOperation({"relay": "inproc", "handle": h, "nbytes": int(buffer.numel() * buffer.element_size())})

    async def get_async(self, metadata, dest=None):
        with _LOCK:
            t = _OBJECTS.pop(metadata["handle"], None)
        if t is None:
            raise KeyError(f"inproc relay handle {metadata['handle']} not found")
        if dest is not None:
            dest.copy_(t)
            t = dest
        return RelayOperation(metadata, result=t)

    def cleanup(self, request_id):
        for h in self._by_request.pop(request_id, []):
            with _LOCK:
                _OBJECTS.pop(h, None)

    def health(self):
        return {"type": "inproc", "ok": True, "live_objects": len(_OBJECTS)}
