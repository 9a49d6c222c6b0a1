"""Builds (and caches per process) the S2-Pro components a stage needs.

With a checkpoint directory: ``config.json`` + safetensors (fish names) for the
dual-AR model, ``tokenizer.json`` for the tokenizer and ``codec.pth`` for the
DAC codec (loaded as in sglang_omni/models/fishaudio_s2_pro/pipeline/stages.py:
38-94).  Without one: random init with fixed seeds and the fallback tokenizer.
``overrides`` shrink the architecture for tests:
{"slow": {...}, "fast": {...}, "s2pro": {"codebook_size": ..}, "dac": {...}}.
"""
from __future__ import annotations

import json
import os
import threading

import torch

from ..weight_loader import has_checkpoint, load_by_prefix
from .codec import DACConfig, DACDecoder, DACEncoder, random_dac_state_dict
from .hf_config import S2ProConfig, config_from_checkpoint
from .model import S2ProDualAR
from .tokenizer import load_s2pro_tokenizer

_LOCK = threading.Lock()
_CACHE: dict[tuple, object] = {}
SEEDS = {"model": 5, "codec": 17}


def _key(model_path, name, device, overrides):
    return (model_path, name, str(device), json.dumps(overrides or {}, sort_keys=True, default=str))


def _ready(obj):
    """Components are built once and then used from several threads, each on its own
    CUDA stream: finish their initialisation before anyone can see them."""
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        torch.cuda.synchronize()
    return obj


def _apply(obj, over: dict | None):
    for k, v in (over or {}).items():
        setattr(obj, k, v)
    return obj


def get_config(model_path: str, overrides: dict | None = None) -> S2ProConfig:
    o = overrides or {}
    cfg = config_from_checkpoint(model_path) if has_checkpoint(model_path) else S2ProConfig()
    _apply(cfg.slow, o.get("slow"))
    _apply(cfg.fast, o.get("fast"))
    _apply(cfg, o.get("s2pro"))
    cfg.fast.vocab_size = cfg.codebook_size
    tok = get_tokenizer(model_path, overrides)
    cfg.semantic_begin_id = tok.convert_tokens_to_ids("<|semantic:0|>")
    cfg.im_end_id = tok.convert_tokens_to_ids("<|im_end|>")
    return cfg


def get_tokenizer(model_path: str, overrides: dict | None = None):
    k = _key(model_path, "tokenizer", "cpu", overrides)
    with _LOCK:
        if k not in _CACHE:
            o = overrides or {}
            vocab = (o.get("slow") or {}).get("vocab_size", 155776)
            cb = (o.get("s2pro") or {}).get("codebook_size", 4096)
            _CACHE[k] = load_s2pro_tokenizer(model_path, vocab, cb)
        return _CACHE[k]


def get_model(model_path: str, device, overrides: dict | None = None) -> S2ProDualAR:
    k = _key(model_path, "model", device, overrides)
    with _LOCK:
        if k in _CACHE:
            return _CACHE[k]
    cfg = get_config(model_path, overrides)
    m = S2ProDualAR(cfg, device)
    if has_checkpoint(model_path):
        m.load_state_dict_fish(load_by_prefix(model_path, ""))
    else:
        m.random_init_(seed=SEEDS["model"])
    _ready(m)
    with _LOCK:
        _CACHE.setdefault(k, m)
        return _CACHE[k]


def dac_config(overrides: dict | None = None) -> DACConfig:
    return _apply(DACConfig(), (overrides or {}).get("dac"))


def get_codec_state(model_path: str, overrides: dict | None = None) -> dict:
    k = _key(model_path, "codec_sd", "cpu", overrides)
    with _LOCK:
        if k in _CACHE:
            return _CACHE[k]
    path = os.path.join(model_path, "codec.pth") if model_path else ""
    if path and os.path.exists(path):
        sd = torch.load(path, map_location="cpu", mmap=True, weights_only=True)
        sd = sd.get("state_dict", sd)
        sd = {kk[len("generator."):] if kk.startswith("generator.") else kk: v for kk, v in sd.items()}
    else:
        sd = random_dac_state_dict(dac_config(overrides), seed=SEEDS["codec"])
    with _LOCK:
        _CACHE.setdefault(k, sd)
        return _CACHE[k]


def get_decoder(model_path: str, device, overrides: dict | None = None) -> DACDecoder:
    k = _key(model_path, "dac_decoder", device, overrides)
    with _LOCK:
        if k in _CACHE:
            return _CACHE[k]
    dec = DACDecoder(dac_config(overrides), device).load_state_dict_dac(get_codec_state(model_path, overrides))
    _ready(dec)
    with _LOCK:
        _CACHE.setdefault(k, dec)
        return _CACHE[k]


def get_encoder(model_path: str, device, overrides: dict | None = None) -> DACEncoder:
    k = _key(model_path, "dac_encoder", device, overrides)
    with _LOCK:
        if k in _CACHE:
            return _CACHE[k]
    enc = DACEncoder(get_codec_state(model_path, overrides), dac_config(overrides), device)
    _ready(enc)
    with _LOCK:
        _CACHE.setdefault(k, enc)
        return _CACHE[k]
