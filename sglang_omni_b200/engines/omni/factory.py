"""Engine factories (sglang_omni/engines/omni/factory.py:35-329): encoder
engines over the generic step engine, AR engines over the paged engine."""
from __future__ import annotations

import torch

from .engine import OmniEngine
from .model_runner import ModelRunner
from .runtime.cache import SimpleCacheManager
from .runtime.common import SimpleResourceManager, SinglePassIterationController
from .runtime.encoder import EncoderBatchPlanner, EncoderInputPreparer, EncoderModelWrapper, EncoderOutputProcessor
from .scheduler import Scheduler


def create_encoder_engine(encode_fn, max_batch_size: int = 32, device="cpu", cache_size: int = 64,
                          gather_window_s: float = 0.008, high_priority: bool = True,
                          explicit_keys: bool = False) -> OmniEngine:
    """Encoders sit on the time-to-first-token/audio path: a short gathering window
    batches a burst of arrivals, and their steps run on a high-priority stream so
    they are not queued behind other stages' decode work on the same GPU.
    ``cache_size`` > 0 keeps that many outputs by request key (``explicit_keys``: only
    requests whose data carries a ``cache_key``; otherwise a hash of their inputs)."""
    sched = Scheduler(EncoderBatchPlanner(max_batch_size, gather_window_s), SimpleResourceManager(max_batch_size * 4),
                      SinglePassIterationController())
    runner = ModelRunner(EncoderModelWrapper(encode_fn), EncoderInputPreparer(), EncoderOutputProcessor(), device)
    prio = None
    if high_priority and torch.device(device).type == "cuda" and torch.cuda.is_available():
        prio = -1   # lower = higher priority; clamped by PyTorch to the device's range
    return OmniEngine(sched, runner, SimpleCacheManager(cache_size, explicit_keys) if cache_size else None,
                      stream_priority=prio, poll_s=0.001)


def create_ar_engine(model, tokenizer=None, max_seq_len: int | None = None, device=None, **kw):
    """AR engine over the paged engine.  ``model``: a ``DecoderLM``, or a transformers causal LM
    (Llama / Mistral / Qwen2 / Qwen3 / Qwen3-MoE), converted first (``models.hf_text``), as the
    reference's factory takes any HF model; ``max_seq_len`` bounds a request's context;
    ``tokenizer`` is accepted for the reference's signature (detokenising happens in the stage)."""
    from ...models.decoder import DecoderLM
    from ..ar import AREngine, KVPool
    from ..ar.adapter import PagedAREngineAdapter

    if max_seq_len is not None:
        kw.setdefault("max_context", int(max_seq_len))
    if not isinstance(model, DecoderLM):
        from ...models.hf_text import decoder_from_hf

        from ...models.hf_text.convert import eos_token_ids

        kw.setdefault("eos_token_ids", eos_token_ids(model))
        model = decoder_from_hf(model, device or "cpu", max_position=kw.get("max_context"))
    cfg = model.cfg
    pages = kw.pop("kv_pages", None) or (kw.get("max_batch", 64) * ((kw.get("max_context", 4096) + 63) // 64) + 8)
    pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, pages, model.embed.device, cfg.dtype)
    return PagedAREngineAdapter(AREngine(model, pool, **kw))
