"""Encoder output cache: LRU keyed by the preprocessing cache key, else a hash
of the request's input tensors (sglang_omni/engines/omni/runtime/cache.py)."""
from __future__ import annotations

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


def cache_key_of(data: Any) -> str:
    if isinstance(data, dict) and data.get("cache_key"):
        return str(data["cache_key"])
    h = hashlib.blake2b(digest_size=16)
    _hash_value(h, data)
    return h.hexdigest()


class SimpleCacheManager:
    def __init__(self, capacity: int = 64):
        self.capacity = capacity
        self._d: OrderedDict[str, Any] = OrderedDict()
        self.hits = 0
        self.misses = 0

    def get(self, request) -> Any | None:
        k = cache_key_of(request.data)
        if k in self._d:
            self._d.move_to_end(k)
            self.hits += 1
            return self._d[k]
        self.misses += 1
        return None

    def put(self, request, output) -> None:
        k = cache_key_of(request.data)
        self._d[k] = output
        self._d.move_to_end(k)
        while len(self._d) > self.capacity:
            self._d.popitem(last=False)
