"""RMSNorm / fused residual-add RMSNorm / LayerNorm (csrc/norm.cu).

Reference counterpart: SGLang RMSNorm with the omni patches,
sglang_omni/vendor/sglang/layers.py:45-87 (HF cast order: normalise in fp32,
round to the input dtype, then multiply by the weight).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext


def rms_norm_ref(x, w, eps):
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (y.to(x.dtype).float() * w.float()).to(x.dtype)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, residual: torch.Tensor | None = None,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """y = rmsnorm(x) * w. With `residual`, first residual += x (in place) and normalise the sum."""
    if not x.is_cuda:
        if residual is not None:
            residual.add_(x)
            x = residual
        y = rms_norm_ref(x, w, eps)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    ext().rmsnorm(x, w, out, residual, eps)
    return out


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None, eps: float = 1e-5,
               out: torch.Tensor | None = None) -> torch.Tensor:
    if not x.is_cuda:
        y = F.layer_norm(x.float(), (x.shape[-1],), w.float(), None if b is None else b.float(), eps).to(x.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    x = x.contiguous()
    if out is None:
        out = torch.empty_like(x)
    ext().layernorm(x, w, b, out, eps)
    return out
