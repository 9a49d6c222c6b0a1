"""Engine factories (sglang_omni/engines/omni/factory.py:35-329): encoder
engines over the generic step engine, AR engines over the paged engine."""
from __future__ import annotations

from .engine import OmniEngine
from .model_runner import ModelRunner
from .runtime.cache import SimpleCacheManager
from .runtime.common import SimpleResourceManager, SinglePassIterationController
from .runtime.encoder import EncoderBatchPlanner, EncoderInputPreparer, EncoderModelWrapper, EncoderOutputProcessor
from .scheduler import Scheduler


def create_encoder_engine(encode_fn, max_batch_size: int = 32, device="cpu", cache_size: int = 64) -> OmniEngine:
    sched = Scheduler(EncoderBatchPlanner(max_batch_size), SimpleResourceManager(max_batch_size * 4),
                      SinglePassIterationController())
    runner = ModelRunner(EncoderModelWrapper(encode_fn), EncoderInputPreparer(), EncoderOutputProcessor(), device)
    return OmniEngine(sched, runner, SimpleCacheManager(cache_size) if cache_size else None)


def create_ar_engine(model, **kw):
    from ..ar import AREngine, KVPool
    from ..ar.adapter import PagedAREngineAdapter

    cfg = model.cfg
    pages = kw.pop("kv_pages", None) or (kw.get("max_batch", 64) * ((kw.get("max_context", 4096) + 63) // 64) + 8)
    pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, pages, model.embed.device, cfg.dtype)
    return PagedAREngineAdapter(AREngine(model, pool, **kw))
