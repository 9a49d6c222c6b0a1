"""Ming-Omni architecture constants and checkpoint-config parsing.

LLM (BailingMoeV2): 32 layers, hidden 4096, 32/4 heads x 128 with QK-norm,
partial RoPE over the first 64 dims (theta 2.4e6), first layer dense (SwiGLU
9216), then MoE with 256 experts top-8 (1024 wide) chosen by sigmoid scores +
expert bias inside the best 4 of 8 groups (group score = sum of its top-2),
renormalised and scaled by 2.5, plus one always-on shared expert; vocab
157184.  Audio tower: Whisper encoder (128 mels, 32 x 1280, 20 heads) +
Conv1d(k3, s2) projection to the LLM width, L2-normalised.
Values as in sglang_omni/models/ming_omni/hf_config.py:10-120.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass

from ..decoder import DecoderConfig


def llm_config(**over) -> DecoderConfig:
    c = DecoderConfig(vocab_size=157184, hidden_size=4096, num_layers=32, num_heads=32, num_kv_heads=4, head_dim=128,
                      intermediate_size=9216, num_experts=256, topk=8, moe_intermediate_size=1024,
                      shared_expert_intermediate_size=1024, shared_expert_gate=False, norm_topk_prob=True,
                      router_mode=1, n_group=8, topk_group=4, routed_scaling_factor=2.5, first_k_dense=1,
                      rms_norm_eps=1e-6, rope_theta=2.4e6, rotary_dim=64, qk_norm=True, max_position=32768,
                      name="ming_bailing_moe_v2")
    for k, v in over.items():
        setattr(c, k, v)
    return c


@dataclass
class WhisperConfig:
    n_mels: int = 128
    n_ctx: int = 15000
    n_state: int = 1280
    n_head: int = 20
    n_layer: int = 32
    ds_kernel_size: int = 3
    ds_stride: int = 2
    mlp_depth: int = 2
    out_dim: int = 4096
    norm_query_embeds: bool = True


EOS_TOKEN_ID = 156895
AUDIO_PATCH = "<audioPatch>"
AUDIO_START = "<audio>"
AUDIO_END = "</audio>"
ROLE_SYSTEM, ROLE_HUMAN, ROLE_ASSISTANT, ROLE_END = "<role>SYSTEM</role>", "<role>HUMAN</role>", \
    "<role>ASSISTANT</role>", "<|role_end|>"


def audio_tokens(mel_frames: int, cfg: WhisperConfig = WhisperConfig()) -> int:
    """Tokens of one audio segment: Whisper's stride-2 conv, then the projection conv
    (sglang_omni/models/ming_omni/components/preprocessor.py:75-93)."""
    n = (mel_frames - 3 + 2) // 2 + 1
    p = cfg.ds_kernel_size // 2
    return (n - cfg.ds_kernel_size + 2 * p) // cfg.ds_stride + 1


def configs_from_hf(model_path: str) -> dict:
    with open(os.path.join(model_path, "config.json")) as f:
        d = json.load(f)
    llm = d.get("llm_config", d)
    m = {"vocab_size": "vocab_size", "hidden_size": "hidden_size", "num_hidden_layers": "num_layers",
         "num_attention_heads": "num_heads", "num_key_value_heads": "num_kv_heads", "head_dim": "head_dim",
         "intermediate_size": "intermediate_size", "num_experts": "num_experts", "num_experts_per_tok": "topk",
         "moe_intermediate_size": "moe_intermediate_size", "rms_norm_eps": "rms_norm_eps",
         "rope_theta": "rope_theta", "n_group": "n_group", "topk_group": "topk_group",
         "routed_scaling_factor": "routed_scaling_factor", "first_k_dense_replace": "first_k_dense",
         "use_qk_norm": "qk_norm", "max_position_embeddings": "max_position"}
    c = llm_config()
    for k, v in m.items():
        if llm.get(k) is not None:
            setattr(c, v, llm[k])
    if llm.get("head_dim") is None:
        c.head_dim = c.hidden_size // c.num_heads
    c.rotary_dim = int(c.head_dim * float(llm.get("partial_rotary_factor", 0.5)))
    c.shared_expert_intermediate_size = int(llm.get("num_shared_experts", 1)) * c.moe_intermediate_size
    a = d.get("audio_config", {})
    w = a.get("whisper_encoder_config", {})
    wc = WhisperConfig(**{k: w[k] for k in ("n_mels", "n_ctx", "n_state", "n_head", "n_layer") if k in w})
    wc.ds_kernel_size = a.get("ds_kernel_size", wc.ds_kernel_size)
    wc.ds_stride = a.get("ds_stride", wc.ds_stride)
    wc.mlp_depth = d.get("mlp_depth", wc.mlp_depth)
    wc.out_dim = c.hidden_size
    wc.norm_query_embeds = a.get("norm_query_embeds", True)
    return {"llm": c, "whisper": wc}
