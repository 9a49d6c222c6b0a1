"""MoE routing, permutation and combine (csrc/fused_ops.cu) + the expert MLP.

``MoEWorkspace`` holds the static buffers of one MoE layer invocation so the
whole expert path (router GEMM -> top-k -> scatter -> grouped w13 (SiLU*up
fused) -> grouped w2 -> combine) runs without host syncs and can be captured
in a CUDA graph.

Reference counterparts: Qwen3-Omni TopK softmax routing + FusedMoE
(sglang_omni/models/qwen3_omni/thinker.py:374-453), the talker's shared
expert with a sigmoid gate (sglang_omni/models/qwen3_omni/talker.py:177-257)
and Ming's sigmoid group-limited routing
(sglang_omni/models/ming_omni/thinker.py:370-462).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext
from .gemm import grouped_linear, linear
from .norm import rms_norm


def route_ref(logits, topk, mode=0, bias=None, n_group=1, topk_group=1, renormalize=True, scaling=1.0):
    logits = logits.float()
    if mode == 0:
        w = torch.softmax(logits, dim=-1)
        sel = w
    else:
        w = torch.sigmoid(logits)
        sel = w + (bias.float() if bias is not None else 0.0)
        if n_group > 1:
            T, E = sel.shape
            g = sel.view(T, n_group, E // n_group)
            gscore = g.topk(2, dim=-1).values.sum(-1)
            keep = gscore.topk(topk_group, dim=-1).indices
            mask = torch.zeros(T, n_group, dtype=torch.bool, device=sel.device)
            mask.scatter_(1, keep, True)
            sel = sel.masked_fill(~mask.repeat_interleave(E // n_group, dim=1), float("-inf"))
    ids = sel.topk(topk, dim=-1).indices
    tw = w.gather(1, ids)
    if renormalize:
        tw = tw / tw.sum(-1, keepdim=True)
    return ids.to(torch.int32), tw * scaling


def moe_ref(x, w_router, w13, w2, topk, renormalize=True, shared=None, mode=0, bias=None, n_group=1, topk_group=1,
            scaling=1.0):
    """Dense fp32 restatement of the routed expert MLP (HF expert loop semantics)."""
    logits = x.float() @ w_router.float().t()
    ids, tw = route_ref(logits, topk, mode, bias, n_group, topk_group, renormalize, scaling)
    I = w13.shape[1] // 2
    out = torch.zeros(x.shape[0], w2.shape[1], dtype=torch.float32, device=x.device)
    for t in range(x.shape[0]):
        for j in range(topk):
            e = int(ids[t, j])
            h = x[t].float() @ w13[e].float().t()
            h = F.silu(h[:I]) * h[I:]
            out[t] += tw[t, j] * (h @ w2[e].float().t())
    if shared is not None:
        sg, s13, s2 = shared
        h = x.float() @ s13.float().t()
        Is = s13.shape[0] // 2
        h = F.silu(h[:, :Is]) * h[:, Is:]
        y = h @ s2.float().t()
        if sg is not None:
            y = torch.sigmoid(x.float() @ sg.float().t()) * y
        out += y
    return out


class MoEWorkspace:
    """Static routing / permutation buffers for up to `max_tokens` tokens."""

    def __init__(self, max_tokens: int, experts: int, topk: int, hidden: int, inter: int, device,
                 dtype=torch.bfloat16):
        self.max_tokens = max_tokens
        rows = max_tokens * topk
        self.logits = torch.empty(max_tokens, experts, dtype=torch.float32, device=device)
        self.topk_ids = torch.empty(max_tokens, topk, dtype=torch.int32, device=device)
        self.topk_w = torch.empty(max_tokens, topk, dtype=torch.float32, device=device)
        self.counts = torch.zeros(experts, dtype=torch.int32, device=device)
        # experts + 1: the last slot is the scatter's done counter; the kernel re-zeroes counts / cursor
        self.cursor = torch.zeros(experts + 1, dtype=torch.int32, device=device)
        self.offsets = torch.zeros(experts + 1, dtype=torch.int32, device=device)
        self.inv_perm = torch.empty(max_tokens, topk, dtype=torch.int32, device=device)
        self.x_perm = torch.empty(rows, hidden, dtype=dtype, device=device)
        self.h_perm = torch.empty(rows, inter, dtype=dtype, device=device)
        self.y_perm = torch.empty(rows, hidden, dtype=dtype, device=device)


def route(logits: torch.Tensor, topk: int, mode: int = 0, bias=None, n_group: int = 1, topk_group: int = 1,
          renormalize: bool = True, scaling: float = 1.0, ws: MoEWorkspace | None = None, x: torch.Tensor | None = None):
    T = logits.shape[0]
    if not logits.is_cuda:
        return route_ref(logits, topk, mode, bias, n_group, topk_group, renormalize, scaling)
    if ws is None:
        ids = torch.empty(T, topk, dtype=torch.int32, device=logits.device)
        tw = torch.empty(T, topk, dtype=torch.float32, device=logits.device)
        ext().moe_route(logits, topk, mode, bias, n_group, topk_group, renormalize, scaling, ids, tw, None, None, None,
                        None, None, None)
        return ids, tw
    ext().moe_route(logits, topk, mode, bias, n_group, topk_group, renormalize, scaling, ws.topk_ids[:T],
                    ws.topk_w[:T], ws.counts, ws.cursor, ws.offsets, ws.inv_perm[:T], x,
                    ws.x_perm[: T * topk] if x is not None else None)
    return ws.topk_ids[:T], ws.topk_w[:T]


def fused_moe(x: torch.Tensor, w_router: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, topk: int,
              ws: MoEWorkspace, renormalize: bool = True, out: torch.Tensor | None = None, mode: int = 0,
              bias=None, n_group: int = 1, topk_group: int = 1, scaling: float = 1.0,
              shared_out: torch.Tensor | None = None, shared_gate: torch.Tensor | None = None,
              norm: tuple | None = None) -> torch.Tensor:
    """Routed expert MLP on the sm_100a kernels: [T, H] -> [T, H].

    ``norm = (residual, weight, eps)`` fuses the next block's add + RMSNorm into
    the combine: residual += moe(x) in place and the normalised rows are returned.
    """
    T, H = x.shape
    E = w13.shape[0]
    if not x.is_cuda:
        y = moe_ref(x, w_router, w13, w2, topk, renormalize, None, mode, bias, n_group, topk_group, scaling)
        if shared_out is not None:
            g = torch.sigmoid(shared_gate.float()) if shared_gate is not None else 1.0
            y = y + g * shared_out.float()
        y = y.to(x.dtype)
        if norm is not None:
            return rms_norm(y, norm[1], norm[2], residual=norm[0], out=out)
        if out is not None:
            out.copy_(y)
            return out
        return y
    logits = ws.logits[:T]
    linear(x, w_router, out=logits)
    route(logits, topk, mode, bias, n_group, topk_group, renormalize, scaling, ws=ws, x=x)
    rows = T * topk
    exp_rows = max(1, rows // E)
    grouped_linear(ws.x_perm[:rows], w13, ws.offsets, gated=True, out=ws.h_perm[:rows], expected_rows=exp_rows)
    grouped_linear(ws.h_perm[:rows], w2, ws.offsets, gated=False, out=ws.y_perm[:rows], expected_rows=exp_rows)
    if out is None:
        out = torch.empty_like(x)
    if norm is not None:
        ext().moe_combine(ws.y_perm[:rows], ws.inv_perm[:T], ws.topk_w[:T], None, shared_out, shared_gate,
                          norm[0], norm[1], out, norm[2])
    else:
        ext().moe_combine(ws.y_perm[:rows], ws.inv_perm[:T], ws.topk_w[:T], out, shared_out, shared_gate)
    return out


def tp_moe(x: torch.Tensor, w_router: torch.Tensor, w13_local: torch.Tensor, w2_local: torch.Tensor, topk: int,
           ws: MoEWorkspace, expert0: int, tp, scatter, renormalize: bool = True, mode: int = 0, bias=None,
           n_group: int = 1, topk_group: int = 1, scaling: float = 1.0, shared_out: torch.Tensor | None = None,
           shared_gate: torch.Tensor | None = None) -> None:
    """Tensor-parallel MoE: every rank routes every token (identical routing on all
    ranks), computes only its experts [expert0, expert0 + El) and the combine stores
    each token's partial sum (local experts + this rank's shared-expert slice) into
    the owner's partial slot (``scatter``) for ``tp.reduce_norm``.  ``x`` is the
    gathered activations; the router GEMM waits for them."""
    T = x.shape[0]
    El = w13_local.shape[0]
    E = ws.offsets.numel() - 1
    logits = ws.logits[:T]
    linear(x, w_router, out=logits, wait=tp.wait)
    rows = T * topk
    ext().moe_route(logits, topk, mode, bias, n_group, topk_group, renormalize, scaling, ws.topk_ids[:T],
                    ws.topk_w[:T], ws.counts, ws.cursor, ws.offsets, ws.inv_perm[:T], x, ws.x_perm[:rows],
                    expert0, El)
    loc = ws.offsets[expert0:expert0 + El + 1]
    exp_rows = max(1, rows // E)
    grouped_linear(ws.x_perm[:rows], w13_local, loc, gated=True, out=ws.h_perm[:rows], expected_rows=exp_rows)
    grouped_linear(ws.h_perm[:rows], w2_local, loc, gated=False, out=ws.y_perm[:rows], expected_rows=exp_rows)
    ext().moe_combine(ws.y_perm[:rows], ws.inv_perm[:T], ws.topk_w[:T], None, shared_out, shared_gate,
                      None, None, None, 1e-6, loc, scatter[0], scatter[1])
