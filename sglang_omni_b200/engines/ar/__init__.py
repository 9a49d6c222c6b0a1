"""Native paged autoregressive engine (replaces the reference's SGLang backend)."""
from .engine import AREngine, ThreadedAREngine
from .kv_pool import KVPool
from .request import ARRequest
from .runner import ARModelRunner

__all__ = ["AREngine", "ThreadedAREngine", "KVPool", "ARRequest", "ARModelRunner"]
