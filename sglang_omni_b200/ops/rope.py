"""QK RMSNorm + RoPE / M-RoPE + paged KV store (csrc/fused_ops.cu).

M-RoPE follows the interleaved THW layout of Qwen3-Omni (transformers
qwen3_omni_moe ``apply_interleaved_mrope``; SGLang MRotaryEmbedding used by
sglang_omni/models/qwen3_omni/thinker.py:223-228); cos/sin tables are rounded
to bf16 like the HF path (and S2-Pro's bf16 RoPE table,
sglang_omni/models/fishaudio_s2_pro/factory.py:57-62).
"""
from __future__ import annotations

import torch

from . import _check
from ._ext import ext


def rope_inv_freq(rot_dim: int, theta: float, scaling: dict | None = None) -> torch.Tensor:
    """Rotation frequencies of the ``rot_dim / 2`` pairs: theta^(-2i / rot_dim), optionally
    rescaled for a longer context than the model was trained at.

    ``scaling`` (the ``rope_scaling`` / ``rope_parameters`` dict of an HF config):
      * ``linear``: every frequency divided by ``factor`` (position interpolation);
      * ``llama3``: the frequency-dependent rule published with Llama 3.1 -- pairs whose
        wavelength (2 pi / f) is shorter than original_context / high_freq_factor keep f,
        those longer than original_context / low_freq_factor get f / factor, and in between
        f is blended between the two with weight s = (original_context / wavelength -
        low_freq_factor) / (high_freq_factor - low_freq_factor) on the unscaled frequency.
    Other kinds (dynamic NTK, YaRN, LongRoPE) are refused."""
    f = 1.0 / (theta ** (torch.arange(0, rot_dim, 2, dtype=torch.int64).float() / rot_dim))
    kind = (scaling or {}).get("rope_type", (scaling or {}).get("type", "default")) if scaling else "default"
    if kind in (None, "default"):
        return f
    factor = float(scaling["factor"])
    if kind == "linear":
        return f / factor
    if kind == "llama3":
        ctx = float(scaling["original_max_position_embeddings"])
        lo, hi = float(scaling.get("low_freq_factor", 1.0)), float(scaling.get("high_freq_factor", 4.0))
        wavelength = 2 * torch.pi / f
        w = ((ctx / wavelength - lo) / (hi - lo)).clamp(0.0, 1.0)   # 0: long wavelength, 1: short
        return w * f + (1.0 - w) * (f / factor)
    raise NotImplementedError(f"RoPE scaling {kind!r} is not supported (default, linear and llama3 are)")


def rope_tables(rot_dim: int, theta: float, max_pos: int, device=None, round_bf16: bool = True,
                scaling: dict | None = None):
    inv_freq = rope_inv_freq(rot_dim, theta, scaling)
    pos = torch.arange(max_pos, dtype=torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    cos, sin = freqs.cos(), freqs.sin()
    if round_bf16:
        cos, sin = cos.bfloat16().float(), sin.bfloat16().float()
    return cos.contiguous().to(device), sin.contiguous().to(device)


def _section_of(j, section, interleaved):
    if interleaved:
        if j % 3 == 1 and j < 3 * section[1]:
            return 1
        if j % 3 == 2 and j < 3 * section[2]:
            return 2
        return 0
    if j < section[0]:
        return 0
    if j < section[0] + section[1]:
        return 1
    return 2


def apply_rope_ref(x, positions, cos_tab, sin_tab, rot_dim, neox=True, section=None, interleaved=True):
    """x: [T, H, D] float. positions: [T] or [3, T]."""
    T, H, D = x.shape
    half = rot_dim // 2
    if positions.dim() == 1:
        pos = positions.long()[None].expand(3, T)
    else:
        pos = positions.long()
    sec_idx = torch.tensor([_section_of(j, section, interleaved) if section is not None else 0 for j in range(half)],
                           device=x.device)
    p = pos[sec_idx]  # [half, T]
    cos = cos_tab[p.t(), torch.arange(half, device=x.device)[None, :]]  # [T, half]
    sin = sin_tab[p.t(), torch.arange(half, device=x.device)[None, :]]
    out = x.clone()
    if neox:
        x1, x2 = x[..., :half], x[..., half:rot_dim]
        out[..., :half] = x1 * cos[:, None] - x2 * sin[:, None]
        out[..., half:rot_dim] = x2 * cos[:, None] + x1 * sin[:, None]
    else:
        x1, x2 = x[..., 0:rot_dim:2], x[..., 1:rot_dim:2]
        out[..., 0:rot_dim:2] = x1 * cos[:, None] - x2 * sin[:, None]
        out[..., 1:rot_dim:2] = x2 * cos[:, None] + x1 * sin[:, None]
    return out


def _rms(x, w, eps, dtype=torch.bfloat16):
    """Per-head RMSNorm with the kernel's rounding points: the normalised value and the
    weighted value are each rounded to the activation dtype (a no-op for fp32)."""
    xf = x.float()
    y = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(dtype).float()
    return (y * w.float()).to(dtype).float()


def qkv_rope_store_ref(qkv, hq, hkv, d, q_norm, k_norm, eps, positions, cos_tab, sin_tab, rot_dim, neox, section,
                       interleaved, slot_mapping, k_cache, v_cache):
    T = qkv.shape[0]
    q = qkv[:, : hq * d].reshape(T, hq, d).float()
    k = qkv[:, hq * d:(hq + hkv) * d].reshape(T, hkv, d).float()
    v = qkv[:, (hq + hkv) * d:(hq + 2 * hkv) * d].reshape(T, hkv, d)
    if q_norm is not None:
        q = _rms(q, q_norm, eps, qkv.dtype)
    if k_norm is not None:
        k = _rms(k, k_norm, eps, qkv.dtype)
    if rot_dim > 0:
        q = apply_rope_ref(q, positions, cos_tab, sin_tab, rot_dim, neox, section, interleaved)
        k = apply_rope_ref(k, positions, cos_tab, sin_tab, rot_dim, neox, section, interleaved)
    qkv[:, : hq * d] = q.reshape(T, -1).to(qkv.dtype)
    qkv[:, hq * d:(hq + hkv) * d] = k.reshape(T, -1).to(qkv.dtype)
    if slot_mapping is not None:
        for t, s in enumerate(slot_mapping.tolist()):
            if s < 0:
                continue
            page, off = s // 64, s % 64
            k_cache[page, :, off] = k[t].to(k_cache.dtype)
            v_cache[page, :, off] = v[t].to(v_cache.dtype)
    return qkv


def qkv_rope_store(qkv: torch.Tensor, num_heads: int, num_kv_heads: int, head_dim: int, positions: torch.Tensor,
                   cos_tab: torch.Tensor, sin_tab: torch.Tensor, rot_dim: int | None = None,
                   q_norm: torch.Tensor | None = None, k_norm: torch.Tensor | None = None, eps: float = 1e-6,
                   neox: bool = True, mrope_section: list[int] | None = None, interleaved: bool = True,
                   slot_mapping: torch.Tensor | None = None, k_cache: torch.Tensor | None = None,
                   v_cache: torch.Tensor | None = None) -> torch.Tensor:
    """In place on qkv [T, (Hq + 2 Hkv) * D]: norm + rotate q, k; store k, v at slot_mapping."""
    rot = head_dim if rot_dim is None else rot_dim
    if not qkv.is_cuda:
        return qkv_rope_store_ref(qkv, num_heads, num_kv_heads, head_dim, q_norm, k_norm, eps, positions, cos_tab,
                                  sin_tab, rot, neox, mrope_section, interleaved, slot_mapping, k_cache, v_cache)
    if _check.enabled():
        _check.check_range("qkv_rope_store", "positions", positions, 0, cos_tab.shape[0])
        if slot_mapping is not None and k_cache is not None:
            _check.check_range("qkv_rope_store", "slot_mapping", slot_mapping, 0, k_cache.shape[0] * 64, allow=-1)
    ext().qkv_rope_store(qkv, num_heads, num_kv_heads, head_dim, q_norm, k_norm, eps, positions,
                         list(mrope_section or [0, 0, 0]), interleaved, cos_tab, sin_tab, rot, neox, slot_mapping,
                         k_cache, v_cache)
    return qkv


def rope_half_inplace(x: torch.Tensor, heads: int, head_stride: int, rot: int, cos: torch.Tensor,
                      sin: torch.Tensor) -> torch.Tensor:
    """In place on ``x`` [rows, cols] bf16: for each of ``heads`` heads (head h at column
    h * head_stride) the first ``rot`` dims rotate by per-row angles, rotate-half style
    (x1, x2) -> (x1 cos - x2 sin, x2 cos + x1 sin) in fp32 -- the vision tower's 2-D
    rotary embedding (transformers' apply_rotary_pos_emb_vision).  cos / sin: fp32 [rows, rot]."""
    if not x.is_cuda:
        v = x.view(x.shape[0], -1)[:, :heads * head_stride].reshape(x.shape[0], heads, head_stride)
        r = v[..., :rot].float()
        h = rot // 2
        rot_half = torch.cat([-r[..., h:], r[..., :h]], -1)
        v[..., :rot] = (r * cos[:, None, :rot] + rot_half * sin[:, None, :rot]).to(x.dtype)
        return x
    ext().rope_half_inplace(x, heads, head_stride, rot, cos, sin)
    return x
