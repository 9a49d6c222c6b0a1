"""Linear layers on the tcgen05 GEMM kernel (csrc/gemm_sm100.cu).

``linear`` is Y = X W^T (+ bias) (+ residual) with an optional fused
activation; ``grouped_linear`` runs one GEMM per group (MoE expert) over
contiguous row ranges given by device offsets, optionally fusing SiLU(gate)*up
when each group's weight stacks [gate; up].

Reference counterparts: the SGLang linear layers and FusedMoE used in
sglang_omni/models/qwen3_omni/thinker.py:192-213,402-412.
"""
from __future__ import annotations

import contextlib
import os
import threading

import torch
import torch.nn.functional as F

from . import _check
from ._ext import ext, status_word

# Per-device split-K scratch of the dense GEMM: fp32 partial sums
# [splits][rows][m_out], reduced by a second kernel.  One buffer per CUDA
# stream: GEMMs of one stream are ordered, those of different engine threads'
# streams may run concurrently.  A graph captured on a stream keeps using that
# stream's buffer on replay (the capture streams are per thread, see
# utils.cuda_graph).  GEMMs needing more than the buffer fall back to no split.
_SPLITK_FLOATS = 8 * 1024 * 1024
_SPLITK_COUNTERS = 1024   # per-tile arrival counters of the in-kernel split-K finalisation
# 3: split-K over a thread-block cluster (partials reduced through distributed shared memory),
# 2: the last split finalises from the global scratch, 1: a second kernel finalises, 0: off
_SPLITK_MODE = int(os.environ.get("OMNI_SPLITK", "3"))
_splitk: dict[tuple[int, int], tuple[torch.Tensor, torch.Tensor]] = {}


def splitk_scratch(device: torch.device):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, torch.cuda.current_stream(idx).cuda_stream)
    sc = _splitk.get(key)
    if sc is None:
        sc = (torch.zeros(_SPLITK_FLOATS, dtype=torch.float32, device=device),
              torch.zeros(_SPLITK_COUNTERS, dtype=torch.int32, device=device))
        _splitk[key] = sc
    return sc

ACT_NONE, ACT_GELU_TANH, ACT_GELU_ERF, ACT_SILU = 0, 1, 2, 3

# Inside ``static_weights()`` the dense GEMM is told that its weight operand is
# not being written by any kernel still in flight on the stream (model
# parameters), so with programmatic dependent launch it fetches its first
# weight tiles while the previous kernel is still running.
_tls = threading.local()


@contextlib.contextmanager
def static_weights():
    prev = getattr(_tls, "static", False)
    _tls.static = True
    try:
        yield
    finally:
        _tls.static = prev
_ACTS = {None: ACT_NONE, "none": ACT_NONE, "gelu_tanh": ACT_GELU_TANH, "gelu_pytorch_tanh": ACT_GELU_TANH,
         "gelu": ACT_GELU_ERF, "gelu_erf": ACT_GELU_ERF, "silu": ACT_SILU}


def act_code(act) -> int:
    if isinstance(act, int):
        return act
    return _ACTS[act]


def _act_ref(y: torch.Tensor, code: int) -> torch.Tensor:
    if code == ACT_GELU_TANH:
        return F.gelu(y, approximate="tanh")
    if code == ACT_GELU_ERF:
        return F.gelu(y)
    if code == ACT_SILU:
        return F.silu(y)
    return y


def linear_ref(x, w, bias=None, residual=None, act=None, out_dtype=None, gated=False):
    """fp32 restatement: the oracle of the kernel and the CPU path."""
    code = act_code(act)
    y = x.float() @ w.float().t()
    if gated:
        i = w.shape[0] // 2
        y = F.silu(y[..., :i]) * y[..., i:]
    if bias is not None:
        y = y + bias.float()
    y = _act_ref(y, code)
    if residual is not None:
        y = y + residual.float()
    return y.to(out_dtype or x.dtype)


def linear(x: torch.Tensor, w: torch.Tensor, bias=None, residual=None, act=None, out=None,
           out_dtype=None, gated: bool = False, scatter=None, wait=None) -> torch.Tensor:
    """Y[..., N] = act(X[..., K] @ W[N, K]^T + bias) + residual.

    With ``gated`` W stacks [gate; up] ([2N, K]) and Y = silu(X W_gate^T) * (X W_up^T).
    Tensor parallel (CUDA only): ``scatter = (peer_ptrs, rows_per)`` stores output
    row r into the owner rank's buffer ``peer_ptrs[r // rows_per] + r * N`` instead of
    ``out``; ``wait = (flags, seq, timeout_s)`` holds the first operand load until
    every flag equals ``seq`` (the gathered activations have arrived).
    """
    if not x.is_cuda:
        y = linear_ref(x, w, bias, residual, act, out_dtype, gated)
        if out is not None:
            out.copy_(y)
            return out
        return y
    n = w.shape[0] // 2 if gated else w.shape[0]
    if out is None:
        out = torch.empty(*x.shape[:-1], n, dtype=out_dtype or torch.bfloat16, device=x.device)
    x2 = x if x.is_contiguous() else x.contiguous()
    rows = x2.numel() // x2.shape[-1]
    ws, ctr = splitk_scratch(x.device)
    if _SPLITK_MODE not in (2, 3):   # 0: no split-K, 1: split-K finalised by a second kernel
        ctr = None
        if _SPLITK_MODE == 0:
            ws = None
    peer, rows_per = scatter if scatter is not None else (None, 0)
    wf, wseq, wt = wait if wait is not None else (None, None, 2.0)
    ext().gemm(w, x2, out, None, n, gated, bias, residual, act_code(act), rows, status_word(x.device), 0, ws, ctr,
               peer, rows_per, wf, wseq, wt, getattr(_tls, "static", False), _SPLITK_MODE == 3)
    return out


def grouped_linear_ref(x, w, offsets, gated=False, out_dtype=None):
    offs = offsets.tolist()
    m_out = w.shape[1] // 2 if gated else w.shape[1]
    out = torch.zeros(x.shape[0], m_out, dtype=torch.float32, device=x.device)
    for g in range(w.shape[0]):
        a, b = offs[g], offs[g + 1]
        if b <= a:
            continue
        y = x[a:b].float() @ w[g].float().t()
        if gated:
            y = F.silu(y[:, :m_out]) * y[:, m_out:]
        out[a:b] = y
    return out.to(out_dtype or x.dtype)


def grouped_linear(x: torch.Tensor, w: torch.Tensor, offsets: torch.Tensor, gated: bool = False, out=None,
                   expected_rows: int | None = None) -> torch.Tensor:
    """Rows offsets[g]:offsets[g+1] of `x` times expert weight w[g] ([G, N, K]).

    With ``gated`` each w[g] is [2I, K] = [gate; up] and the result is
    silu(x w_gate^T) * (x w_up^T), shape [rows, I].
    """
    if not x.is_cuda:
        y = grouped_linear_ref(x, w, offsets, gated)
        if out is not None:
            out.copy_(y)
            return out
        return y
    m_out = w.shape[1] // 2 if gated else w.shape[1]
    if out is None:
        out = torch.empty(x.shape[0], m_out, dtype=torch.bfloat16, device=x.device)
    if expected_rows is None:
        expected_rows = max(1, x.shape[0] // max(1, w.shape[0]))
    if _check.enabled():
        _check.check_offsets("grouped_linear", offsets, x.shape[0])
    ext().gemm(w, x, out, offsets, m_out, gated, None, None, ACT_NONE, expected_rows, status_word(x.device))
    return out
