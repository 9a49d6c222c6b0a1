"""Encoder output cache: LRU keyed by the preprocessing cache key, else a hash
of the request's input tensors (sglang_omni/engines/omni/runtime/cache.py)."""
from __future__ import annotations

import dataclasses
import hashlib
from collections import OrderedDict
from typing import Any

import torch


def _hash_value(h, v: Any):
    if isinstance(v, torch.Tensor):
        t = v.detach().contiguous().cpu()
        h.update(str((t.dtype, tuple(t.shape))).encode())
        h.update(t.view(torch.uint8).numpy().tobytes() if t.numel() else b"")
    elif isinstance(v, dict):
        for k in sorted(v):
            h.update(str(k).encode())
            _hash_value(h, v[k])
    elif isinstance(v, (list, tuple)):
        for x in v:
            _hash_value(h, x)
    else:
        h.update(repr(v).encode())


def explicit_key(data: Any) -> str | None:
    """The key the request's producer attached (a ``cache_key`` entry or attribute), if any."""
    k = data.get("cache_key") if isinstance(data, dict) else getattr(data, "cache_key", None)
    return str(k) if k else None


def cache_key_of(data: Any) -> str:
    k = explicit_key(data)
    if k is not None:
        return k
    h = hashlib.blake2b(digest_size=16)
    if dataclasses.is_dataclass(data) and not isinstance(data, type):
        data = {f.name: getattr(data, f.name) for f in dataclasses.fields(data)}
    _hash_value(h, data)
    return h.hexdigest()


class SimpleCacheManager:
    """LRU of ``capacity`` outputs.  ``explicit_only``: only requests that carry a key of their
    own (preprocessing's media keys) take part; the rest are encoded every time, without hashing
    their inputs."""

    def __init__(self, capacity: int = 64, explicit_only: bool = False):
        self.capacity = capacity
        self.explicit_only = explicit_only
        self._d: OrderedDict[str, Any] = OrderedDict()
        self.hits = 0
        self.misses = 0

    def _key(self, request) -> str | None:
        return explicit_key(request.data) if self.explicit_only else cache_key_of(request.data)

    def get(self, request) -> Any | None:
        k = self._key(request)
        if k is None:
            return None
        if k in self._d:
            self._d.move_to_end(k)
            self.hits += 1
            return self._d[k]
        self.misses += 1
        return None

    def put(self, request, output) -> None:
        k = self._key(request)
        if k is None or output is None:
            return
        self._d[k] = output
        self._d.move_to_end(k)
        while len(self._d) > self.capacity:
            self._d.popitem(last=False)
