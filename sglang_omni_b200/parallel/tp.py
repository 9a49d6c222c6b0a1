"""Tensor parallelism over NVLink peer memory.

One process per GPU; every rank of the group runs the same tokens.  Attention
heads are split (column-parallel QKV, row-parallel o_proj), the MoE experts are
split (each rank computes its experts for every token) and the two reduce
points of a layer are fused kernels instead of all-reduce calls:

  row-parallel GEMM / MoE combine   epilogue stores output row r straight into
                                    the part[rank] slot of r's owner rank
                                    (``r // rows_per``): the reduce-scatter's
                                    transfer happens inside the producing kernel;
  ``tp_reduce_norm``                the owner sums the world partial rows, adds
                                    the residual, RMS-normalises with the next
                                    block's weight and stores the normalised row
                                    into every rank's ``gath`` (the all-gather);
  next GEMM                         waits on the phase-B flags before its first
                                    TMA load (``wait=``), then reads ``gath``.

The residual stream is kept by the owners (each rank updates the rows it owns);
``gather_residual`` also all-gathers the residual rows where a caller needs the
full hidden state (captured layers).  Sequence numbers live on the device, so
a decode step with every layer's exchanges is one CUDA graph.

Reference counterparts (call sites only, ``tp_size`` is forced to 1 there):
sglang_omni/models/qwen3_omni/thinker.py:167-213 (QKV / o_proj split),
:447-453 (MoE all-reduce), sglang_omni/vendor/sglang/layers.py:92-137
(all-reduce + residual + RMSNorm fusion).
"""
from __future__ import annotations

import torch

from ..ops._ext import ext, status_word
from .hostgroup import barrier, rank_of, world_of
from .symm import RegionLayout, SymmetricBuffer


class TPGroup:
    def __init__(self, hidden: int, max_tokens: int, device, group=None, dtype=torch.bfloat16,
                 timeout_s: float = 2.0):
        self.group = group
        self.rank = rank_of(group)
        self.world = world_of(group)
        self.hidden, self.max_tokens = hidden, max_tokens
        self.device = torch.device(device)
        self.timeout_s = timeout_s
        row_bytes = max_tokens * hidden * 2
        lay = RegionLayout()
        lay.add("flags", 2 * self.world * 4)
        lay.add("part", self.world * row_bytes)
        lay.add("gath", row_bytes)
        lay.add("gres", row_bytes)
        self.buf = SymmetricBuffer(lay.size, group, self.device)
        o = lay.offsets
        base = self.buf.peers
        # [4, world]: part / gath / gres / flags bases of every rank
        table = [[b + o["part"] for b in base], [b + o["gath"] for b in base], [b + o["gres"] for b in base],
                 [b + o["flags"] for b in base]]
        self.ptrs = torch.tensor(table, dtype=torch.int64, device=self.device)
        # where this rank's partial rows go: owner d's part slot [rank]
        self.scatter_ptrs = torch.tensor([b + o["part"] + self.rank * row_bytes for b in base], dtype=torch.int64,
                                         device=self.device)
        self.gath = self.buf.view(o["gath"], (max_tokens, hidden), dtype)
        self.gres = self.buf.view(o["gres"], (max_tokens, hidden), dtype)
        self.part_local = self.buf.view(o["part"] + self.rank * row_bytes, (max_tokens, hidden), dtype)
        self.flags_b = self.buf.view(o["flags"] + self.world * 4, (self.world,), torch.int32)
        self.buf.view(o["flags"], (2 * self.world,), torch.int32).zero_()
        self.seq = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.counter = torch.zeros(1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        barrier(group)

    # ------------------------------------------------------------ geometry
    def rows_per(self, tokens: int) -> int:
        return max(1, (tokens + self.world - 1) // self.world)

    def owned(self, tokens: int) -> tuple[int, int]:
        rp = self.rows_per(tokens)
        a = min(tokens, self.rank * rp)
        return a, min(tokens, a + rp)

    @property
    def wait(self):
        """``wait=`` argument of ``ops.linear`` for a GEMM that reads ``gath``."""
        return (self.flags_b, self.seq, self.timeout_s)

    def scatter(self, tokens: int):
        """``scatter=`` argument: output rows go to their owners' partial slots."""
        assert tokens <= self.max_tokens, f"{tokens} tokens > TP buffer capacity {self.max_tokens}"
        return (self.scatter_ptrs, self.rows_per(tokens))

    # ------------------------------------------------------------ reduce point
    def reduce_norm(self, residual: torch.Tensor, norm_w: torch.Tensor, eps: float, tokens: int,
                    gather_residual: bool = False, single_src: bool = False,
                    local_only: bool = False) -> torch.Tensor:
        """Sums the partials of the owned rows + residual (updated in place on the owned
        rows), RMSNorm, all-gather.  Returns ``gath[:tokens]`` (read it only through a
        GEMM given ``wait=self.wait``, or after :meth:`wait_gather`).

        ``single_src``: the owned rows were already reduced into ``part_local`` (an
        expert-parallel combine); ``local_only``: the normalised owned rows stay on this
        rank (``gath[owned]``, read in stream order) instead of being all-gathered."""
        ext().tp_reduce_norm(self.ptrs, self.rank, self.world, tokens, self.rows_per(tokens), self.max_tokens,
                             residual, norm_w, eps, gather_residual, self.seq, self.counter,
                             status_word(self.device), self.timeout_s, single_src, local_only)
        return self.gath[:tokens]

    def wait_gather(self):
        """Stream-ordered wait for the last reduce point's all-gather (for non-GEMM readers)."""
        ext().tp_wait(self.ptrs, self.rank, self.world, self.seq, self.counter, status_word(self.device),
                      self.timeout_s)

    def close(self):
        self.buf.close()


def head_split(num_heads: int, num_kv_heads: int, rank: int, world: int) -> tuple[range, range]:
    """Query heads and KV heads a rank keeps.  With fewer KV heads than ranks the KV
    heads are replicated: rank r keeps KV head r * Hkv // world, whose query group
    contains r's query heads."""
    assert num_heads % world == 0, "query heads must divide over the TP group"
    hq = num_heads // world
    q = range(rank * hq, (rank + 1) * hq)
    if num_kv_heads >= world:
        assert num_kv_heads % world == 0
        hk = num_kv_heads // world
        kv = range(rank * hk, (rank + 1) * hk)
    else:
        assert world % num_kv_heads == 0
        kv = range(rank * num_kv_heads // world, rank * num_kv_heads // world + 1)
    group = num_heads // num_kv_heads
    assert q.start // group == kv.start and (q.stop - 1) // group == kv.stop - 1, "query heads outside the KV group"
    return q, kv
