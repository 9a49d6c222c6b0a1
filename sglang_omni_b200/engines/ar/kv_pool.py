"""Paged KV pool: one tensor [layers, 2, pages, Hkv, 64, D] and a page allocator.

Page 0 is reserved as the padding page of CUDA-graph decode buckets.
The allocator is the native ``_runtime.PageAllocator`` when built, else a
Python free list with the same interface.

With ``enable_prefix_cache()`` the pool also keeps a page-granular radix
tree of finished requests' KV (``_runtime.PrefixCache``): a new request whose
prompt starts with cached full pages reuses them instead of recomputing
them, and cached pages that no request references are evicted (LRU, leaves
first) whenever an allocation would otherwise fail.

Reference counterpart: SGLang's token-to-KV pool behind
sglang_omni/engines/ar/sglang_backend/model_worker.py (mem_fraction_static
sizing, sglang_omni/engines/ar/sglang_backend/server_args_builder.py:10-35).
"""
from __future__ import annotations

import torch

try:
    from ... import _runtime as _rt
except ImportError:  # pragma: no cover
    _rt = None

PAGE = 64


class _PyAllocator:
    def __init__(self, num_pages: int, reserved: int = 1):
        self._n = num_pages
        self._free = list(range(num_pages - 1, reserved - 1, -1))

    def num_free(self):
        return len(self._free)

    def num_pages(self):
        return self._n

    def can_alloc(self, n):
        return n <= len(self._free)

    def alloc(self, n):
        if n > len(self._free):
            raise RuntimeError("KV pool out of pages")
        out = self._free[len(self._free) - n:]
        del self._free[len(self._free) - n:]
        return out[::-1]

    def alloc_one(self):
        return self._free.pop() if self._free else -1

    def free(self, pages):
        self._free.extend(pages)


class KVPool:
    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, num_pages: int, device,
                 dtype=torch.bfloat16):
        self.device = torch.device(device)
        self.num_layers = num_layers
        self.num_pages = num_pages
        self.kv = torch.zeros(num_layers, 2, num_pages, num_kv_heads, PAGE, head_dim, dtype=dtype, device=self.device)
        self._alloc = _rt.PageAllocator(num_pages, 1) if _rt is not None else _PyAllocator(num_pages, 1)
        self.prefix_cache = None

    def enable_prefix_cache(self):
        if _rt is None:
            raise RuntimeError("the prefix cache needs the native _runtime extension")
        if self.prefix_cache is None:
            self.prefix_cache = _rt.PrefixCache(PAGE)
        return self.prefix_cache

    @classmethod
    def for_memory(cls, num_layers, num_kv_heads, head_dim, bytes_budget: int, device, dtype=torch.bfloat16,
                   max_pages: int | None = None):
        per_page = num_layers * 2 * num_kv_heads * PAGE * head_dim * torch.finfo(dtype).bits // 8
        pages = max(2, int(bytes_budget // per_page))
        if max_pages is not None:
            pages = min(pages, max_pages)
        return cls(num_layers, num_kv_heads, head_dim, pages, device, dtype)

    def allocator_native(self):
        return self._alloc

    @property
    def free_pages(self) -> int:
        return self._alloc.num_free()

    def can_alloc(self, n: int) -> bool:
        if self._alloc.can_alloc(n):
            return True
        pc = self.prefix_cache
        return pc is not None and self._alloc.num_free() + pc.evictable_pages() >= n

    def ensure_free(self, n: int) -> bool:
        """Makes at least n pages free in the allocator itself (evicting cached
        prefixes if needed), for callers that allocate through it directly."""
        short = n - self._alloc.num_free()
        if short > 0 and self.prefix_cache is not None:
            self._alloc.free(self.prefix_cache.evict(short))
        return self._alloc.can_alloc(n)

    def alloc(self, n: int) -> list[int]:
        self.ensure_free(n)
        return list(self._alloc.alloc(n))

    def free(self, pages: list[int]):
        if pages:
            self._alloc.free(list(pages))

    @staticmethod
    def pages_for(tokens: int) -> int:
        return (tokens + PAGE - 1) // PAGE
