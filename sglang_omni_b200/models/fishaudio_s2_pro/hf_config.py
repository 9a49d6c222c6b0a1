"""FishAudio S2-Pro (dual-AR TTS) architecture constants and checkpoint-config parsing.

Slow AR (text model): Qwen3-style dense decoder, 36 layers, hidden 2560,
SwiGLU 9728, 32/8 heads x 128, vocab 155776, tied embeddings, QK-norm,
non-neox (pairwise) RoPE with theta 1e6 (defaults of S2ProSGLangTextModel,
sglang_omni/models/fishaudio_s2_pro/sglang_model.py:163-181).
Fast AR (audio decoder): 4 layers predicting codebooks 1..9 after the
semantic token, codebook vocab 4096, 10 codebooks
(FishQwen3AudioDecoder, .../text2semantic/modeling.py:919-1010).  The fast
AR's shape is read from the checkpoint's config.json when one is present;
the random-init default is 4 layers x 1024 (16 x 64 heads, SwiGLU 3072), so
``project_in`` maps the 2560-wide slow hidden state to 1024.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import torch

from ..decoder import DecoderConfig


def slow_config(**over) -> DecoderConfig:
    c = DecoderConfig(vocab_size=155776, hidden_size=2560, num_layers=36, num_heads=32, num_kv_heads=8, head_dim=128,
                      intermediate_size=9728, rms_norm_eps=1e-6, rope_theta=1e6, rope_neox=False, qk_norm=True,
                      tie_word_embeddings=True, max_position=32768, name="s2pro_slow_ar")
    for k, v in over.items():
        setattr(c, k, v)
    return c


def fast_config(**over) -> DecoderConfig:
    c = DecoderConfig(vocab_size=4096, hidden_size=1024, num_layers=4, num_heads=16, num_kv_heads=8, head_dim=64,
                      intermediate_size=3072, rms_norm_eps=1e-6, rope_theta=1e6, rope_neox=False, qk_norm=True,
                      tie_word_embeddings=False, max_position=16, name="s2pro_fast_ar")
    for k, v in over.items():
        setattr(c, k, v)
    return c


@dataclass
class S2ProConfig:
    slow: DecoderConfig = field(default_factory=slow_config)
    fast: DecoderConfig = field(default_factory=fast_config)
    num_codebooks: int = 10
    codebook_size: int = 4096
    # token ids (fallback tokenizer layout; a checkpoint's tokenizer overrides them)
    semantic_begin_id: int = 151678
    im_end_id: int = 151645

    @property
    def semantic_end_id(self) -> int:
        return self.semantic_begin_id + self.codebook_size - 1

    @property
    def vq_scale(self) -> float:
        return (self.num_codebooks + 1) ** -0.5


def _fish_to_decoder(d: dict, base: DecoderConfig) -> DecoderConfig:
    """FishQwen3Config keys (.../text2semantic/configuration.py:86-200) -> DecoderConfig."""
    m = {"vocab_size": "vocab_size", "dim": "hidden_size", "n_layer": "num_layers", "n_head": "num_heads",
         "n_local_heads": "num_kv_heads", "head_dim": "head_dim", "intermediate_size": "intermediate_size",
         "rope_base": "rope_theta", "norm_eps": "rms_norm_eps", "attention_qk_norm": "qk_norm",
         "tie_word_embeddings": "tie_word_embeddings"}
    for k, v in m.items():
        if d.get(k) is not None:
            setattr(base, v, d[k])
    if base.num_kv_heads in (-1, None):
        base.num_kv_heads = base.num_heads
    if not d.get("head_dim"):
        base.head_dim = base.hidden_size // base.num_heads
    return base


def config_from_checkpoint(model_path: str, dtype=torch.bfloat16) -> S2ProConfig:
    with open(os.path.join(model_path, "config.json")) as f:
        d = json.load(f)
    tc = d.get("text_config", d)
    ac = d.get("audio_decoder_config") or {}
    cfg = S2ProConfig()
    cfg.slow = _fish_to_decoder(tc, slow_config(dtype=dtype))
    cfg.slow.max_position = int(tc.get("max_seq_len", cfg.slow.max_position))
    cfg.fast = _fish_to_decoder(ac, fast_config(dtype=dtype))
    cfg.num_codebooks = int(ac.get("num_codebooks", cfg.num_codebooks))
    cfg.codebook_size = int(ac.get("vocab_size", cfg.codebook_size))
    cfg.fast.vocab_size = cfg.codebook_size
    cfg.fast.max_position = cfg.num_codebooks + 6
    cfg.fast.tie_word_embeddings = False
    return cfg
