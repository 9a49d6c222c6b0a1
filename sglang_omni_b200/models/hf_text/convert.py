"""Hugging Face causal LMs -> ``DecoderLM`` (fused layouts, the sm_100a kernels on a GPU).

The reference serves arbitrary transformers models through its generic AR engine
(``create_ar_engine(model=AutoModelForCausalLM...)``, sglang_omni/engines/omni/factory.py and
examples/run_openai_llama_server.py:198-229) and runs them with HF's own forward.  Here the
weights move into the one decoder implementation of this package, so a Llama / Mistral / Qwen2 /
Qwen3 / Qwen3-MoE model gets the paged KV cache, chunked prefill, CUDA-graph decode and the
tcgen05 GEMM / attention kernels like the omni models do.

Covered configuration fields: GQA heads and head_dim, q / k / v biases (Qwen2; Llama's
``attention_bias``), per-head q / k RMSNorm (Qwen3), RoPE theta with linear or Llama-3 frequency
scaling, tied embeddings, softmax top-k routed experts with optional top-k renormalisation and
dense ``mlp_only_layers`` / ``decoder_sparse_step`` layers (Qwen3-MoE).  Refused with a message:
sliding-window attention (Mistral v0.1 style, Qwen2 ``use_sliding_window``), MLP biases, other
RoPE scalings."""
from __future__ import annotations

import json
import os
from typing import Any

import torch

from ..decoder import DecoderConfig, DecoderLM
from ..weight_loader import load_by_prefix, load_decoder_from_hf

SUPPORTED_ARCHITECTURES = ("LlamaForCausalLM", "MistralForCausalLM", "Qwen2ForCausalLM", "Qwen3ForCausalLM",
                           "Qwen3MoeForCausalLM")


def _get(c, name, default=None):
    return c.get(name, default) if isinstance(c, dict) else getattr(c, name, default)


def _rope(c) -> tuple[float, dict | None]:
    params = _get(c, "rope_parameters") or {}
    scaling = _get(c, "rope_scaling") or None
    theta = _get(c, "rope_theta") or params.get("rope_theta") or 10000.0
    if scaling is None and params.get("rope_type", "default") not in (None, "default"):
        scaling = params
    return float(theta), (dict(scaling) if scaling else None)


def decoder_config_from_hf(c: Any, dtype: torch.dtype = torch.bfloat16, max_position: int | None = None) -> DecoderConfig:
    """``c``: a transformers ``PretrainedConfig`` or its ``config.json`` dict."""
    archs = list(_get(c, "architectures") or [])
    arch = archs[0] if archs else ""
    if arch and arch not in SUPPORTED_ARCHITECTURES:
        raise ValueError(f"architecture {arch!r} is not one of {SUPPORTED_ARCHITECTURES}")
    heads = int(_get(c, "num_attention_heads"))
    hidden = int(_get(c, "hidden_size"))
    layers = int(_get(c, "num_hidden_layers"))
    win = _get(c, "sliding_window")
    if win and (_get(c, "use_sliding_window", arch != "Qwen2ForCausalLM") and int(win) < int(
            max_position or _get(c, "max_position_embeddings") or 0)):
        raise NotImplementedError(f"{arch}: sliding-window attention ({win}) is not supported by the paged engine")
    if _get(c, "mlp_bias", False):
        raise NotImplementedError(f"{arch}: MLP biases are not supported")
    theta, scaling = _rope(c)
    from ...ops.rope import rope_inv_freq

    rope_inv_freq(2, theta, scaling)      # refuses unsupported scalings before any weight is read
    qwen2 = arch == "Qwen2ForCausalLM" or _get(c, "model_type") == "qwen2"
    qwen3 = arch.startswith("Qwen3") or str(_get(c, "model_type", "")).startswith("qwen3")
    kw = dict(vocab_size=int(_get(c, "vocab_size")), hidden_size=hidden, num_layers=layers, num_heads=heads,
              num_kv_heads=int(_get(c, "num_key_value_heads") or heads),
              head_dim=int(_get(c, "head_dim") or hidden // heads),
              intermediate_size=int(_get(c, "intermediate_size") or 0),
              rms_norm_eps=float(_get(c, "rms_norm_eps", 1e-6)), rope_theta=theta, rope_scaling=scaling,
              rope_neox=True, qk_norm=qwen3, attention_bias=bool(qwen2 or _get(c, "attention_bias", False)),
              tie_word_embeddings=bool(_get(c, "tie_word_embeddings", False)),
              max_position=int(max_position or _get(c, "max_position_embeddings") or 32768), dtype=dtype,
              name=(arch or "hf_causal_lm").lower())
    experts = int(_get(c, "num_experts") or 0)
    if experts:
        step = int(_get(c, "decoder_sparse_step") or 1)
        dense = set(int(i) for i in (_get(c, "mlp_only_layers") or []))
        dense |= {i for i in range(layers) if (i + 1) % step != 0}
        kw.update(num_experts=experts, topk=int(_get(c, "num_experts_per_tok")),
                  moe_intermediate_size=int(_get(c, "moe_intermediate_size")),
                  norm_topk_prob=bool(_get(c, "norm_topk_prob", True)), router_mode=0,
                  mlp_only_layers=tuple(sorted(dense)))
    return DecoderConfig(**kw)


def eos_token_ids(src: Any) -> tuple[int, ...]:
    """End-of-sequence ids of a checkpoint directory (generation_config.json, else config.json) or
    of a transformers model (its generation / model config)."""
    found = None
    if isinstance(src, str):
        for name in ("generation_config.json", "config.json"):
            path = os.path.join(src, name)
            if os.path.exists(path):
                with open(path) as f:
                    found = json.load(f).get("eos_token_id")
                if found is not None:
                    break
    else:
        gen = getattr(src, "generation_config", None)
        found = getattr(gen, "eos_token_id", None) if gen is not None else None
        if found is None:
            found = getattr(getattr(src, "config", None), "eos_token_id", None)
    if found is None:
        return ()
    return tuple(int(x) for x in (found if isinstance(found, (list, tuple)) else [found]))


@torch.no_grad()
def decoder_from_hf(src: Any, device="cpu", dtype: torch.dtype | None = None,
                    max_position: int | None = None) -> DecoderLM:
    """``src``: a transformers causal-LM module (its config and state dict are read) or a local
    checkpoint directory (config.json + safetensors).  ``dtype`` defaults to bf16 on a GPU and to
    the checkpoint's dtype (fp32 for a module) on the CPU."""
    dev = torch.device(device)
    if isinstance(src, str):
        with open(os.path.join(src, "config.json")) as f:
            c = json.load(f)
        sd = load_by_prefix(src, "")
        ck = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}.get(
            str(c.get("torch_dtype") or c.get("dtype") or "bfloat16"), torch.bfloat16)
    else:
        c = src.config
        sd = src.state_dict()
        ck = next(src.parameters()).dtype
    if dtype is None:
        dtype = torch.bfloat16 if dev.type == "cuda" else ck
    cfg = decoder_config_from_hf(c, dtype, max_position)
    model = DecoderLM(cfg, device=dev)
    load_decoder_from_hf(model, sd, "model.", "lm_head.weight")
    return model
