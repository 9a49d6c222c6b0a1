"""Convolutions and activations of the audio encoders and vocoders, channels-
last ([B, T, C]).  Convolutions run as tcgen05 GEMMs over im2col rows
(csrc/audio_ops.cu + csrc/gemm_sm100.cu); transposed convolutions as one GEMM
plus an overlap-add; depthwise convs and Snake activations as elementwise
kernels.  CPU tensors use PyTorch restatements (the oracles).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext
from .gemm import linear


def snake(x: torch.Tensor, alpha: torch.Tensor, beta: torch.Tensor | None = None, log_scale: bool = True,
          out: torch.Tensor | None = None) -> torch.Tensor:
    """SnakeBeta (log_scale: alpha/beta are log-parameters) or Snake1d (beta=None, alpha linear)."""
    if not x.is_cuda:
        a = alpha.float()
        b = (beta if beta is not None else alpha).float()
        if log_scale:
            a, b = a.exp(), b.exp()
        xf = x.float()
        y = xf + (1.0 / (b + 1e-9)) * torch.sin(xf * a) ** 2
        return y.to(x.dtype)
    x = x.contiguous()
    if out is None:
        out = torch.empty_like(x)
    ext().snake(x, alpha.float().contiguous(), None if beta is None else beta.float().contiguous(), out, log_scale)
    return out


def causal_conv1d(x: torch.Tensor, w2d: torch.Tensor, bias: torch.Tensor | None, kernel: int, dilation: int = 1,
                  stride: int = 1, pad_left: int | None = None, t_out: int | None = None,
                  residual: torch.Tensor | None = None, act=None) -> torch.Tensor:
    """x [B, T, Cin]; w2d [Cout, K*Cin] in (tap, channel) order -> [B, T_out, Cout].

    Default padding is causal: (K-1)*dil - (stride-1) on the left (HF CausalConvNet); positions
    past the input on either side read zeros, so ``pad_left`` + ``t_out`` also express symmetric
    padding.  ``act`` ("gelu" / "silu") runs in the GEMM epilogue."""
    B, T, C = x.shape
    eff = (kernel - 1) * dilation + 1
    if pad_left is None:
        pad_left = eff - stride
    if t_out is None:
        t_out = (T + pad_left - eff) // stride + 1
        # HF adds right padding so the last (partial) frame is produced
        if (T + pad_left - eff) % stride != 0:
            t_out += 1
    if not x.is_cuda:
        xp = F.pad(x.float().transpose(1, 2), (pad_left, max(0, (t_out - 1) * stride + eff - T - pad_left)))
        w = w2d.float().view(w2d.shape[0], kernel, C).permute(0, 2, 1)
        y = F.conv1d(xp, w, None if bias is None else bias.float(), stride=stride, dilation=dilation)
        y = y.transpose(1, 2)[:, :t_out]
        if act == "gelu":
            y = F.gelu(y)
        elif act == "silu":
            y = F.silu(y)
        if residual is not None:
            y = y + residual.float()
        return y.to(x.dtype)
    if kernel == 1 and stride == 1 and pad_left == 0:
        cols = x.contiguous()
    else:
        cols = torch.empty(B, t_out, kernel * C, dtype=x.dtype, device=x.device)
        ext().conv1d_im2col(x.contiguous(), cols, kernel, dilation, stride, pad_left)
    return linear(cols, w2d, bias=bias, residual=residual, act=act)


def conv_transpose1d(x: torch.Tensor, w_t: torch.Tensor, bias: torch.Tensor | None, stride: int,
                     trim_left: int | None = None, t_out: int | None = None) -> torch.Tensor:
    """Transposed conv with kernel 2*stride, trimmed: output sample u is sample u + trim_left of
    the full (T + 1) * stride result.

    Defaults (trim ``stride`` on both sides -> [B, (T-1)*stride, Cout]) match the Code2Wav
    CausalTransConvNet; DAC's causal variant keeps the left edge (trim_left=0, t_out=T*stride).
    w_t: [(2s)*Cout, Cin] = the ConvTranspose1d weight [Cin, Cout, 2s] permuted to ((j, o), c)."""
    B, T, C = x.shape
    Cout = w_t.shape[0] // (2 * stride)
    shift = stride if trim_left is None else trim_left
    if t_out is None:
        t_out = (T - 1) * stride if trim_left is None else (T + 1) * stride - shift
    if not x.is_cuda:
        w = w_t.float().view(2 * stride, Cout, C).permute(2, 1, 0)  # [Cin, Cout, 2s]
        y = F.conv_transpose1d(x.float().transpose(1, 2), w, None if bias is None else bias.float(), stride=stride)
        y = y[..., shift: shift + t_out]
        return y.transpose(1, 2).to(x.dtype).contiguous()
    cols = linear(x.contiguous(), w_t)  # [B, T, 2s*Cout]
    out = torch.empty(B, t_out, Cout, dtype=x.dtype, device=x.device)
    ext().conv_transpose_ola(cols, bias, out, stride, shift)
    return out


def dwconv1d_causal(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """Depthwise causal conv: w [C, K] -> [B, T, C]."""
    B, T, C = x.shape
    K = w.shape[1]
    if not x.is_cuda:
        xp = F.pad(x.float().transpose(1, 2), (K - 1, 0))
        y = F.conv1d(xp, w.float().view(C, 1, K), None if bias is None else bias.float(), groups=C)
        return y.transpose(1, 2).to(x.dtype)
    out = torch.empty_like(x)
    ext().dwconv1d_causal(x.contiguous(), w.float().contiguous(), None if bias is None else bias.float(), out)
    return out


def conv2d(x: torch.Tensor, w2d: torch.Tensor, bias: torch.Tensor | None, k: int, stride: int, pad: int,
           act=None) -> torch.Tensor:
    """x [N, H, W, C]; w2d [O, k*k*C] in (kh, kw, c) order -> [N, Ho, Wo, O]."""
    N, H, W, C = x.shape
    Ho = (H + 2 * pad - k) // stride + 1
    Wo = (W + 2 * pad - k) // stride + 1
    if not x.is_cuda:
        w = w2d.float().view(w2d.shape[0], k, k, C).permute(0, 3, 1, 2)
        y = F.conv2d(x.float().permute(0, 3, 1, 2), w, None if bias is None else bias.float(), stride=stride,
                     padding=pad)
        y = y.permute(0, 2, 3, 1)
        if act == "gelu":
            y = F.gelu(y)
        return y.to(x.dtype).contiguous()
    Kc = k * k * C
    Kp = (Kc + 7) // 8 * 8  # 16-byte rows for TMA
    cols = torch.zeros(N, Ho, Wo, Kp, dtype=x.dtype, device=x.device) if Kp != Kc else \
        torch.empty(N, Ho, Wo, Kc, dtype=x.dtype, device=x.device)
    ext().conv2d_im2col(x.contiguous(), cols, k, k, stride, pad)
    if Kp != Kc:
        w2d = F.pad(w2d, (0, Kp - Kc))
    return linear(cols, w2d, bias=bias, act=act)
