"""HF safetensors loading by key prefix, and the HF -> fused-layout mapping of
the decoder weights.

Checkpoints load unchanged: tensors are read (memory-mapped) from every
``*.safetensors`` shard (or the shards listed in ``model.safetensors.index.json``),
filtered by prefix (``thinker.``, ``thinker.audio_tower.``, ``talker.``,
``talker.code_predictor.``, ``code2wav.``...) with the prefix stripped, then
fused into this framework's layouts (q/k/v -> qkv, gate/up -> w13 per expert,
expert stacks).  Accepts both per-expert keys
(``mlp.experts.{e}.gate_proj.weight``) and pre-stacked ones
(``mlp.experts.gate_up_proj``).

Reference counterparts: sglang_omni/models/weight_loader.py:16-266 and the
fused-weight remaps of sglang_omni/models/qwen3_omni/thinker.py:747-827,
talker.py:955-1027.
"""
from __future__ import annotations

import glob
import json
import os
from typing import Iterator

import torch

from .decoder import DecoderLM


def has_checkpoint(model_path: str | None) -> bool:
    return bool(model_path) and os.path.isdir(model_path) and bool(
        glob.glob(os.path.join(model_path, "*.safetensors")))


def _shards(model_path: str) -> list[str]:
    idx = os.path.join(model_path, "model.safetensors.index.json")
    if os.path.exists(idx):
        with open(idx) as f:
            files = sorted(set(json.load(f)["weight_map"].values()))
        return [os.path.join(model_path, x) for x in files]
    return sorted(glob.glob(os.path.join(model_path, "*.safetensors")))


def iter_tensors(model_path: str, prefix: str = "") -> Iterator[tuple[str, torch.Tensor]]:
    from safetensors import safe_open

    for shard in _shards(model_path):
        with safe_open(shard, framework="pt") as f:
            for k in f.keys():
                if k.startswith(prefix):
                    yield k[len(prefix):], f.get_tensor(k)


def load_by_prefix(model_path: str, prefix: str) -> dict[str, torch.Tensor]:
    return dict(iter_tensors(model_path, prefix))


@torch.no_grad()
def load_decoder_from_hf(model: DecoderLM, sd: dict[str, torch.Tensor], model_prefix: str = "model.",
                         lm_head_key: str | None = "lm_head.weight", embed_key: str = "embed_tokens.weight") -> None:
    """Fills a DecoderLM from HF-named tensors (prefix of the text model already stripped)."""
    cfg = model.full_cfg if hasattr(model, "full_cfg") else model.cfg
    g = lambda k: sd[model_prefix + k]  # noqa: E731
    cp = lambda dst, src: dst.copy_(src.to(dst.dtype))  # noqa: E731
    sh = getattr(model, "shard", lambda kind, t: t)   # tensor parallel: this rank's slice
    if model_prefix + embed_key in sd:
        cp(model.embed, g(embed_key))
    for i, L in enumerate(model.layers):
        p = f"layers.{i}."
        cp(L.ln1, g(p + "input_layernorm.weight"))
        cp(L.ln2, g(p + "post_attention_layernorm.weight"))
        if model_prefix + p + "self_attn.qkv_proj.weight" in sd:
            cp(L.qkv, sh("qkv", g(p + "self_attn.qkv_proj.weight")))
        else:
            cp(L.qkv, sh("qkv", torch.cat([g(p + f"self_attn.{n}_proj.weight") for n in "qkv"], 0)))
        cp(L.o, sh("o", g(p + "self_attn.o_proj.weight")))
        if getattr(cfg, "attention_bias", False):
            cp(L.qkv_bias, sh("qkv_bias", torch.cat([g(p + f"self_attn.{n}_proj.bias") for n in "qkv"], 0)))
        if cfg.qk_norm:
            cp(L.q_norm, g(p + "self_attn.q_norm.weight"))
            cp(L.k_norm, g(p + "self_attn.k_norm.weight"))
        if cfg.is_moe_layer(i):
            cp(L.router, g(p + "mlp.gate.weight"))
            stacked = model_prefix + p + "mlp.experts.gate_up_proj"
            e0, El = getattr(model, "expert0", 0), L.w13.shape[0]   # this rank's experts (expert parallel)
            if stacked in sd:
                cp(L.w13, sd[stacked][e0:e0 + El])
                cp(L.w2, g(p + "mlp.experts.down_proj")[e0:e0 + El])
            else:
                for j in range(El):
                    q = p + f"mlp.experts.{e0 + j}."
                    L.w13[j].copy_(torch.cat([g(q + "gate_proj.weight"), g(q + "up_proj.weight")], 0).to(L.w13.dtype))
                    L.w2[j].copy_(g(q + "down_proj.weight").to(L.w2.dtype))
            if hasattr(L, "router_bias") and model_prefix + p + "mlp.gate.e_score_correction_bias" in sd:
                cp(L.router_bias, g(p + "mlp.gate.e_score_correction_bias"))
            if cfg.shared_expert_intermediate_size:
                s = p + "mlp.shared_expert."
                cp(L.s13, sh("s13", torch.cat([g(s + "gate_proj.weight"), g(s + "up_proj.weight")], 0)))
                cp(L.s2, sh("s2", g(s + "down_proj.weight")))
                if cfg.shared_expert_gate:
                    cp(L.sgate, g(p + "mlp.shared_expert_gate.weight"))
        else:
            cp(L.mlp13, sh("mlp13", torch.cat([g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")], 0)))
            cp(L.mlp2, sh("mlp2", g(p + "mlp.down_proj.weight")))
    cp(model.final_norm, g("norm.weight"))
    if model.lm_head is not None and lm_head_key is not None and lm_head_key in sd:
        cp(model.lm_head, sh("lm_head", sd[lm_head_key]))


def export_decoder_to_hf(model: DecoderLM, model_prefix: str = "model.") -> dict[str, torch.Tensor]:
    """Inverse of load_decoder_from_hf (per-expert keys); used for round-trip tests and checkpoint export."""
    cfg = model.cfg
    out: dict[str, torch.Tensor] = {model_prefix + "embed_tokens.weight": model.embed.detach().clone()}
    q, kv = cfg.q_size, cfg.kv_size
    for i, L in enumerate(model.layers):
        p = model_prefix + f"layers.{i}."
        out[p + "input_layernorm.weight"] = L.ln1.clone()
        out[p + "post_attention_layernorm.weight"] = L.ln2.clone()
        out[p + "self_attn.q_proj.weight"] = L.qkv[:q].clone()
        out[p + "self_attn.k_proj.weight"] = L.qkv[q:q + kv].clone()
        out[p + "self_attn.v_proj.weight"] = L.qkv[q + kv:].clone()
        if hasattr(L, "qkv_bias"):
            out[p + "self_attn.q_proj.bias"] = L.qkv_bias[:q].clone()
            out[p + "self_attn.k_proj.bias"] = L.qkv_bias[q:q + kv].clone()
            out[p + "self_attn.v_proj.bias"] = L.qkv_bias[q + kv:].clone()
        out[p + "self_attn.o_proj.weight"] = L.o.clone()
        if cfg.qk_norm:
            out[p + "self_attn.q_norm.weight"] = L.q_norm.clone()
            out[p + "self_attn.k_norm.weight"] = L.k_norm.clone()
        if cfg.is_moe_layer(i):
            out[p + "mlp.gate.weight"] = L.router.clone()
            I = cfg.moe_intermediate_size
            for e in range(cfg.num_experts):
                out[p + f"mlp.experts.{e}.gate_proj.weight"] = L.w13[e, :I].clone()
                out[p + f"mlp.experts.{e}.up_proj.weight"] = L.w13[e, I:].clone()
                out[p + f"mlp.experts.{e}.down_proj.weight"] = L.w2[e].clone()
            if cfg.shared_expert_intermediate_size:
                Is = cfg.shared_expert_intermediate_size
                out[p + "mlp.shared_expert.gate_proj.weight"] = L.s13[:Is].clone()
                out[p + "mlp.shared_expert.up_proj.weight"] = L.s13[Is:].clone()
                out[p + "mlp.shared_expert.down_proj.weight"] = L.s2.clone()
                if cfg.shared_expert_gate:
                    out[p + "mlp.shared_expert_gate.weight"] = L.sgate.clone()
        else:
            I = cfg.intermediate_size
            out[p + "mlp.gate_proj.weight"] = L.mlp13[:I].clone()
            out[p + "mlp.up_proj.weight"] = L.mlp13[I:].clone()
            out[p + "mlp.down_proj.weight"] = L.mlp2.clone()
    out[model_prefix + "norm.weight"] = model.final_norm.clone()
    if model.lm_head is not None:
        out["lm_head.weight"] = model.lm_head.clone()
    return out
