"""Qwen3-Omni-30B-A3B architecture constants and HF-config parsing.

Defaults follow the published Qwen3-Omni-30B-A3B-Instruct config (thinker
text: 48 layers, hidden 2048, 32/4 heads x 128, 128 experts top-8, moe 768,
vocab 151936, M-RoPE [24, 20, 20] interleaved, theta 1e6; talker: 20 layers,
hidden 1024, 16/2 heads, 128 experts top-6, moe 384 + shared 768, codec vocab
3072; code predictor: 5 layers, 16/8 heads, MLP 3072, 16 code groups x 2048).
The reference keeps the same values in sglang_omni/config/qwen3_omni.py:6-328.
"""
from __future__ import annotations

import json
import os

from ..decoder import DecoderConfig

AUDIO_TOKEN_ID = 151646
IMAGE_TOKEN_ID = 151655
VIDEO_TOKEN_ID = 151656
AUDIO_START_TOKEN_ID = 151647
VISION_START_TOKEN_ID = 151652
THINKER_EOS_IDS = (151645, 151643)  # <|im_end|>, <|endoftext|>


def thinker_text_config(**over) -> DecoderConfig:
    c = DecoderConfig(vocab_size=151936, hidden_size=2048, num_layers=48, num_heads=32, num_kv_heads=4, head_dim=128,
                      intermediate_size=768, num_experts=128, topk=8, moe_intermediate_size=768, norm_topk_prob=True,
                      rms_norm_eps=1e-6, rope_theta=1e6, mrope_section=[24, 20, 20], mrope_interleaved=True,
                      qk_norm=True, max_position=65536, name="qwen3_omni_thinker")
    for k, v in over.items():
        setattr(c, k, v)
    return c


def talker_text_config(**over) -> DecoderConfig:
    c = DecoderConfig(vocab_size=3072, hidden_size=1024, num_layers=20, num_heads=16, num_kv_heads=2, head_dim=128,
                      intermediate_size=2048, num_experts=128, topk=6, moe_intermediate_size=384,
                      shared_expert_intermediate_size=768, shared_expert_gate=True, norm_topk_prob=True,
                      rms_norm_eps=1e-6, rope_theta=1e6, mrope_section=[24, 20, 20], mrope_interleaved=True,
                      qk_norm=True, max_position=65536, name="qwen3_omni_talker")
    for k, v in over.items():
        setattr(c, k, v)
    return c


def code_predictor_config(**over) -> DecoderConfig:
    c = DecoderConfig(vocab_size=2048, hidden_size=1024, num_layers=5, num_heads=16, num_kv_heads=8, head_dim=128,
                      intermediate_size=3072, rms_norm_eps=1e-6, rope_theta=1e6, qk_norm=True, max_position=64,
                      name="qwen3_omni_code_predictor")
    for k, v in over.items():
        setattr(c, k, v)
    return c


def _text_cfg_from_hf(d: dict, base: DecoderConfig) -> DecoderConfig:
    m = {"vocab_size": "vocab_size", "hidden_size": "hidden_size", "num_hidden_layers": "num_layers",
         "num_attention_heads": "num_heads", "num_key_value_heads": "num_kv_heads", "head_dim": "head_dim",
         "intermediate_size": "intermediate_size", "num_experts": "num_experts", "num_experts_per_tok": "topk",
         "moe_intermediate_size": "moe_intermediate_size", "norm_topk_prob": "norm_topk_prob",
         "rms_norm_eps": "rms_norm_eps", "rope_theta": "rope_theta",
         "shared_expert_intermediate_size": "shared_expert_intermediate_size"}
    for k, attr in m.items():
        if k in d and d[k] is not None:
            setattr(base, attr, d[k])
    rs = d.get("rope_scaling") or d.get("rope_parameters") or {}
    if isinstance(rs, dict):
        if "mrope_section" in rs:
            base.mrope_section = list(rs["mrope_section"])
        if "rope_theta" in rs:
            base.rope_theta = rs["rope_theta"]
        if "interleaved" in rs or "mrope_interleaved" in rs:
            base.mrope_interleaved = bool(rs.get("interleaved", rs.get("mrope_interleaved", True)))
    if d.get("mlp_only_layers"):
        base.mlp_only_layers = tuple(d["mlp_only_layers"])
    return base


def load_hf_config(model_path: str) -> dict:
    p = os.path.join(model_path, "config.json")
    with open(p) as f:
        return json.load(f)


def configs_from_hf(model_path: str) -> dict[str, DecoderConfig]:
    d = load_hf_config(model_path)
    out = {}
    th = d.get("thinker_config", {})
    out["thinker"] = _text_cfg_from_hf(th.get("text_config", {}), thinker_text_config())
    tk = d.get("talker_config", {})
    if tk:
        out["talker"] = _text_cfg_from_hf(tk.get("text_config", {}), talker_text_config())
        cp = tk.get("code_predictor_config", {})
        out["code_predictor"] = _text_cfg_from_hf(cp, code_predictor_config())
    return out
