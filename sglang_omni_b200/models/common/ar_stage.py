"""Generic autoregressive text stage: an EngineExecutor over the paged engine.

The payload's data carries ``prompt_token_ids`` (or ``input_ids``); sampling
comes from ``request.params['sampling']`` overridden by
``request.params['stage_sampling'][<stage>]``; streaming emits per-token text
deltas; the result carries token ids, text, finish reason and usage.
"""
from __future__ import annotations

from typing import Any

import torch

from ...engines.ar import AREngine, ARRequest, KVPool
from ...engines.ar.adapter import PagedAREngineAdapter
from ...executors import EngineExecutor
from ...proto import StagePayload
from ...sampling_params import SamplingParams
from .tokenizer import IncrementalDetokenizer


def sampling_for(payload: StagePayload, stage: str) -> SamplingParams:
    params = payload.request.params or {}
    base = dict(params.get("sampling") or {})
    per = (params.get("stage_sampling") or {}).get(stage) or {}
    base.update(per)
    return SamplingParams.from_dict(base)


def prompt_ids_of(data: Any) -> list[int]:
    if isinstance(data, dict):
        for k in ("prompt_token_ids", "input_ids", "token_ids"):
            if k in data and data[k] is not None:
                v = data[k]
                return v.tolist() if isinstance(v, torch.Tensor) else list(v)
    if isinstance(data, (list, tuple)):
        return list(data)
    raise ValueError("payload has no prompt token ids")


def create_ar_executor(model, stage_name: str, tokenizer, max_batch: int = 64, max_context: int = 4096,
                       max_prefill_tokens: int = 8192, kv_pages: int | None = None, use_graphs: bool = True,
                       eos_token_ids=(), default_max_new_tokens: int = 128, prefix_cache: bool = True,
                       rank_group=None) -> EngineExecutor:
    """``rank_group``: a ``parallel.rank_group.GroupSpec`` (builder, mode, world, GPUs); the stage is
    then served by that group (this process is its leader) and ``model`` is ignored."""
    dev = model.embed.device if model is not None else (torch.device("cuda", torch.cuda.current_device())
                                                        if rank_group is not None and rank_group.gpus
                                                        else torch.device("cpu"))
    pages = kv_pages or (max_batch * ((max_context + 63) // 64) + 8)
    engine_args = dict(max_batch=max_batch, max_prefill_tokens=max_prefill_tokens, max_context=max_context,
                       use_graphs=use_graphs and dev.type == "cuda", eos_token_ids=tuple(eos_token_ids),
                       prefix_cache=prefix_cache)
    if rank_group is not None:
        from ...parallel.rank_group import GroupedAREngine, StageRankGroup

        rank_group.engine_args = engine_args
        rank_group.kv_pages = pages
        rg = StageRankGroup(rank_group)
        engine = rg.start()
        adapter = PagedAREngineAdapter(engine, threaded=GroupedAREngine(engine, rg))
    else:
        cfg = model.cfg
        pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, pages, dev, cfg.dtype)
        engine = AREngine(model, pool, **engine_args)
        adapter = PagedAREngineAdapter(engine)
    detoks: dict[str, IncrementalDetokenizer] = {}

    def request_builder(payload: StagePayload) -> ARRequest:
        sp = sampling_for(payload, stage_name)
        ids = prompt_ids_of(payload.data)
        detoks[payload.request_id] = IncrementalDetokenizer(tokenizer)
        return ARRequest(rid=payload.request_id, prompt_ids=ids, sampling=sp,
                         max_new_tokens=sp.max_new_tokens or default_max_new_tokens)

    def stream_builder(payload: StagePayload, chunk):
        tok, _info = chunk
        d = detoks.get(payload.request_id)
        text = d.push(tok) if d is not None else ""
        return {"modality": "text", "token_ids": [int(tok)], "text": text}

    def result_builder(payload: StagePayload, r: ARRequest) -> StagePayload:
        detoks.pop(payload.request_id, None)
        text = tokenizer.decode(r.output_ids, skip_special_tokens=True)
        data = {"token_ids": list(r.output_ids), "text": text, "finish_reason": r.finish_reason,
                "usage": {"prompt_tokens": len(r.prompt_ids), "completion_tokens": len(r.output_ids),
                          "total_tokens": len(r.prompt_ids) + len(r.output_ids)}}
        return StagePayload(payload.request_id, payload.request, data)

    ex = EngineExecutor(adapter, request_builder, result_builder, stream_builder)
    ex.ar_engine = engine
    return ex
