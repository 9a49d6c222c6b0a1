"""Expert-parallel MoE over NVLink peer memory.

Each rank of the EP group owns ``experts / world`` consecutive experts and runs
attention on its own tokens (data-parallel attention).  One MoE layer:

  1. route locally (gate GEMM + top-k kernel);
  2. ``ep_counts``: per-expert counts of every rank are exchanged through the
     symmetric buffer; every rank derives the same row offsets;
  3. ``ep_dispatch``: every (token, k) row is stored directly into its expert
     owner's receive buffer, already in expert-major order (the permutation of
     a local MoE and the all-to-all in one kernel), then a flag barrier;
  4. the owner runs its two grouped GEMMs (gate/up with SiLU*up in the
     epilogue, then down) over the received rows;
  5. ``ep_combine``: every expert-output row is stored back into its source
     rank's slot, flag barrier, and the source does the top-k weighted sum
     (+ gated shared expert) with ``moe_combine``.

All steps are device-side (no host synchronisation), so a decode step with
its 48 MoE layers is captured in one CUDA graph.  The reference only has
SGLang's EP/all-reduce call sites, never enabled
(sglang_omni/models/qwen3_omni/thinker.py:402-453).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import route
from ..ops._ext import ext, status_word
from ..ops.gemm import grouped_linear, linear
from .symm import RegionLayout, SymmetricBuffer


class EPMoE:
    def __init__(self, experts: int, topk: int, hidden: int, inter: int, max_tokens: int, device,
                 group=None, dtype=torch.bfloat16, cap_rows: int | None = None, timeout_s: float = 2.0):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        assert experts % self.world == 0, "experts must divide evenly over the EP group"
        self.experts, self.topk, self.hidden, self.inter = experts, topk, hidden, inter
        self.local_experts = experts // self.world
        self.max_tokens = max_tokens
        self.max_slots = max_tokens * topk
        self.cap_rows = cap_rows or self.world * self.max_slots
        self.device = torch.device(device)
        self.timeout_s = timeout_s
        lay = RegionLayout()
        lay.add("counts", self.world * experts * 4)
        lay.add("flags", 3 * self.world * 4)
        lay.add("recv_x", self.cap_rows * hidden * 2)
        lay.add("recv_meta", self.cap_rows * 2 * 4)
        lay.add("comb", self.max_slots * hidden * 2)
        self.layout = lay
        self.buf = SymmetricBuffer(lay.size, group, self.device)
        o = lay.offsets
        self.offs = [o["counts"], o["flags"], o["recv_x"], o["recv_meta"], o["comb"]]
        self.recv_x = self.buf.view(o["recv_x"], (self.cap_rows, hidden), dtype)
        self.comb = self.buf.view(o["comb"], (self.max_slots, hidden), dtype)
        dev = self.device
        self.cursor = torch.zeros(experts, dtype=torch.int32, device=dev)
        self.local_offsets = torch.zeros(self.local_experts + 1, dtype=torch.int32, device=dev)
        self.total_rows = torch.zeros(1, dtype=torch.int32, device=dev)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        self.h_perm = torch.empty(self.cap_rows, inter, dtype=dtype, device=dev)
        self.y_perm = torch.empty(self.cap_rows, hidden, dtype=dtype, device=dev)
        self.slots = torch.arange(self.max_slots, dtype=torch.int32, device=dev)

    def _common(self, ids):
        return (ids, self.buf.peer_base, self.offs, self.rank, self.world, self.experts)

    def forward(self, x: torch.Tensor, w_router: torch.Tensor, w13_local: torch.Tensor, w2_local: torch.Tensor,
                renormalize: bool = True, mode: int = 0, bias=None, n_group: int = 1, topk_group: int = 1,
                scaling: float = 1.0, shared_out: torch.Tensor | None = None,
                shared_gate: torch.Tensor | None = None, out: torch.Tensor | None = None,
                norm: tuple | None = None) -> torch.Tensor:
        """x [T, H] (this rank's tokens) -> [T, H]; w13_local / w2_local hold this rank's experts.

        ``norm = (residual, weight, eps)``: residual += result in place and the
        RMS-normalised rows are returned (the next block's fused add + norm)."""
        T = x.shape[0]
        assert T <= self.max_tokens, f"{T} tokens > EP buffer capacity {self.max_tokens}"
        st = status_word(x.device)
        logits = linear(x, w_router, out_dtype=torch.float32)
        ids, w = route(logits, self.topk, mode, bias, n_group, topk_group, renormalize, scaling)
        e = ext()
        ids_c = ids.contiguous()
        e.ep_counts(ids_c, self.buf.peer_base, self.offs, self.rank, self.world, self.experts, self.hidden,
                    self.cap_rows, self.max_slots, self.cursor, self.local_offsets, self.total_rows, self.epoch, st,
                    self.timeout_s)
        e.ep_dispatch(x.contiguous(), ids_c, self.buf.peer_base, self.offs, self.rank, self.world, self.experts,
                      self.cap_rows, self.max_slots, self.cursor, self.local_offsets, self.total_rows, self.epoch, st,
                      self.timeout_s)
        exp_rows = max(1, (T * self.topk * self.world) // self.experts)
        grouped_linear(self.recv_x, w13_local, self.local_offsets, gated=True, out=self.h_perm,
                       expected_rows=exp_rows)
        grouped_linear(self.h_perm, w2_local, self.local_offsets, gated=False, out=self.y_perm,
                       expected_rows=exp_rows)
        e.ep_combine(self.y_perm, ids_c, self.buf.peer_base, self.offs, self.rank, self.world, self.experts,
                     self.cap_rows, self.max_slots, self.cursor, self.local_offsets, self.total_rows, self.epoch, st,
                     self.timeout_s)
        if out is None:
            out = torch.empty_like(x)
        n = T * self.topk
        if norm is not None:
            e.moe_combine(self.comb[:n], self.slots[:n].view(T, self.topk), w, None, shared_out, shared_gate,
                          norm[0], norm[1], out, norm[2])
        else:
            e.moe_combine(self.comb[:n], self.slots[:n].view(T, self.topk), w, out, shared_out, shared_gate)
        return out

    def close(self):
        self.buf.close()
