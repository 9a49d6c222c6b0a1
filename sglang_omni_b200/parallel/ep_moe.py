"""Expert-parallel MoE over NVLink peer memory.

Each rank of the EP group owns ``experts / world`` consecutive experts and runs
attention on its own tokens (data-parallel attention).  One MoE layer is four
kernels after the router GEMM and top-k, with the two cross-rank waits inside
the kernels that consume the data:

  1. ``ep_dispatch``: every (token, k) row is stored straight into its expert
     owner's receive segment for that expert (a CTA reserves its rows of an
     expert with one system-scope atomic on the owner's counter, so no count
     exchange comes first); the last CTA raises this rank's dispatch flag on
     every peer;
  2. the gated w13 grouped GEMM (tcgen05, SiLU*up in the epilogue) waits for
     every source's dispatch flag, reads the final per-expert counts and runs
     over the received segments (local memory, TMA);
  3. the w2 grouped GEMM's epilogue stores each output row into the ``comb``
     slot of the rank the row came from (over NVLink), then raises this rank's
     combine flag on every peer;
  4. ``moe_combine`` waits for every owner's combine flag, then does the top-k
     weighted sum (+ the next block's residual add + RMSNorm).

All steps are device-side (no host synchronisation, sequence numbers on the
device), so a decode step with its 48 MoE layers is one CUDA graph.  Every rank
must run every layer (the flags are collective).  The reference only has
SGLang's EP / all-reduce call sites, never enabled
(sglang_omni/models/qwen3_omni/thinker.py:402-453).
"""
from __future__ import annotations

import torch

from ..ops._ext import ext, status_word
from ..ops.gemm import linear
from .hostgroup import barrier, rank_of, world_of
from .symm import RegionLayout, SymmetricBuffer


class EPMoE:
    def __init__(self, experts: int, topk: int, hidden: int, inter: int, max_tokens: int, device,
                 group=None, dtype=torch.bfloat16, timeout_s: float = 2.0):
        self.group = group
        self.rank = rank_of(group)
        self.world = world_of(group)
        assert experts % self.world == 0, "experts must divide evenly over the EP group"
        self.experts, self.topk, self.hidden, self.inter = experts, topk, hidden, inter
        self.local_experts = El = experts // self.world
        self.max_tokens = max_tokens
        self.max_slots = max_tokens * topk
        # an expert receives at most one row per token of every rank
        self.seg_cap = self.world * max_tokens
        self.device = dev = torch.device(device)
        self.timeout_s = timeout_s
        lay = RegionLayout()
        lay.add("flags", 2 * self.world * 4)
        lay.add("cursor", El * 4)
        lay.add("recv_x", El * self.seg_cap * hidden * 2)
        lay.add("recv_tag", El * self.seg_cap * 2 * 4)
        lay.add("comb", self.max_slots * hidden * 2)
        self.layout = lay
        self.buf = SymmetricBuffer(lay.size, group, dev)
        o = lay.offsets
        self.offs = [o["flags"], o["cursor"], o["recv_x"], o["recv_tag"], o["comb"]]
        self.flags = self.buf.view(o["flags"], (2, self.world), torch.int32)
        self.cursor = self.buf.view(o["cursor"], (El,), torch.int32)
        self.recv_x = self.buf.view(o["recv_x"], (El * self.seg_cap, hidden), dtype)
        self.recv_tag = self.buf.view(o["recv_tag"], (El * self.seg_cap, 2), torch.int32)
        self.comb = self.buf.view(o["comb"], (self.max_slots, hidden), dtype)
        with torch.cuda.device(dev):
            self.flags.zero_()
            self.cursor.zero_()
            torch.cuda.synchronize(dev)
        barrier(group)
        peers = self.buf.peers
        r, w = self.rank, self.world
        # where this rank raises its combine flag on every peer: flags[1][r] (the dispatch kernel
        # derives flags[0][r] from the buffer bases itself)
        self.sig_combine = torch.tensor([b + o["flags"] + 4 * (w + r) for b in peers], dtype=torch.int64, device=dev)
        self.peer_comb = torch.tensor([b + o["comb"] for b in peers], dtype=torch.int64, device=dev)
        self.seq = torch.zeros(1, dtype=torch.int32, device=dev)
        self.arrive = torch.zeros(2, dtype=torch.int32, device=dev)   # dispatch CTAs, w2 CTAs
        self.seg_counts = torch.zeros(El, dtype=torch.int32, device=dev)
        self.h_seg = torch.empty(El * self.seg_cap, inter, dtype=dtype, device=dev)
        self.slots = torch.arange(self.max_slots, dtype=torch.int32, device=dev)
        self.topk_ids = torch.empty(max_tokens, topk, dtype=torch.int32, device=dev)
        self.topk_w = torch.empty(max_tokens, topk, dtype=torch.float32, device=dev)
        # timing hook: a list that receives a name after each launch (the caller records an event)
        self._marks = None

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
        e = ext()
        mark = self._marks.append if self._marks is not None else (lambda _n: None)
        logits = linear(x, w_router, out_dtype=torch.float32)
        mark("router")
        ids, w = self.topk_ids[:T], self.topk_w[:T]
        e.moe_route(logits, self.topk, mode, bias, n_group, topk_group, renormalize, scaling, ids, w, None, None,
                    None, None, None, None, 0, 0)
        mark("topk")
        x = x.contiguous()
        e.ep_dispatch(x, ids, self.buf.peer_base, self.offs, self.rank, self.world, self.experts, self.seg_cap,
                      self.seq, self.arrive[0:1], st)
        mark("dispatch")
        exp_rows = max(1, (T * self.topk * self.world) // self.experts)
        e.gemm_ep(w13_local, self.recv_x, self.h_seg, self.inter, True, self.seg_cap, self.cursor, self.seg_counts,
                  self.flags[0], self.seq, self.timeout_s, None, None, 0, None, None, None, None, exp_rows, st)
        mark("w13 (waits for dispatch)")
        e.gemm_ep(w2_local, self.h_seg, self.comb, self.hidden, False, self.seg_cap, self.seg_counts, None,
                  None, None, self.timeout_s, self.recv_tag, self.peer_comb, self.max_slots, self.sig_combine,
                  self.seq, self.arrive[1:2], self.cursor, exp_rows, st)
        mark("w2 + combine stores")
        if out is None:
            out = torch.empty_like(x)
        n = T * self.topk
        wait = dict(wait_flags=self.flags[1], wait_seq=self.seq, status=st, timeout_s=self.timeout_s)
        if norm is not None:
            e.moe_combine(self.comb[:n], self.slots[:n].view(T, self.topk), w, None, shared_out, shared_gate,
                          norm[0], norm[1], out, norm[2], **wait)
        else:
            e.moe_combine(self.comb[:n], self.slots[:n].view(T, self.topk), w, out, shared_out, shared_gate, **wait)
        mark("top-k sum (waits for owners)")
        return out

    def close(self):
        self.buf.close()
