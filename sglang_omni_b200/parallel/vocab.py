"""Vocab-parallel LM head sampling over NVLink peer memory.

Under tensor parallelism every rank holds a slice of the LM head's rows, so a
rank computes only logits columns ``[vocab0, vocab0 + vocab_local)``.  Instead
of all-gathering the full fp32 logits (rows x vocab x 4 bytes onto every rank),
``VocabParallelSampler`` reduces each rank's slice to a small record per row
(max, sum of exp, the slice's greedy / Gumbel-max winner and its top-``cand``
(value, token) pairs) and stores it into every rank's exchange region from the
kernel that computed it (csrc/vocab_parallel.cu).  Every rank then draws the
same token from the records:

* greedy rows, temperature-only rows and rows with ``top_k <= cand`` (with or
  without top-p / min-p on top) draw exactly the token of the single-GPU sampler;
* top-p / min-p rows without such a top-k are exact when the final threshold
  lies above every rank's ``cand``-th value; otherwise (flat distributions, the
  kept set larger than the union of candidates) they draw from the union and
  are counted in ``inexact_rows``.  A larger ``cand`` (up to 256) widens the union.

Reference counterpart: the thinker's vocab-parallel LM head and logits
all-gather (sglang_omni/models/qwen3_omni/thinker.py:614-619, sglang
ParallelLMHead + LogitsProcessor), with tp_size forced to 1 there.
"""
from __future__ import annotations

import torch

from ..ops._ext import ext, status_word
from ..ops.sampling import SamplingTensors
from .hostgroup import barrier, rank_of, world_of
from .symm import RegionLayout, SymmetricBuffer

MAX_CAND = 256
MAX_WORLD = 8
HEADER_BYTES = 32


def vocab_slice(vocab: int, rank: int, world: int) -> tuple[int, int, int]:
    """(vocab0, vocab_local, padded width) of a rank's LM-head rows: equal slices of
    ceil(vocab / world) rows (a multiple of 16 for the GEMM), the last one shorter."""
    width = (vocab + world - 1) // world
    width = (width + 15) // 16 * 16
    v0 = min(vocab, rank * width)
    return v0, max(0, min(width, vocab - v0)), width


class VocabParallelSampler:
    """Collective construction: every rank of ``group`` builds one with the same sizes."""

    def __init__(self, vocab: int, max_rows: int, device, group=None, cand: int = 64, timeout_s: float = 2.0):
        self.group = group
        self.rank, self.world = rank_of(group), world_of(group)
        assert 1 <= self.world <= MAX_WORLD, f"vocab-parallel sampling supports up to {MAX_WORLD} ranks"
        assert 1 <= cand <= MAX_CAND
        self.vocab, self.max_rows, self.cand = vocab, max_rows, cand
        self.vocab0, self.vocab_local, self.width = vocab_slice(vocab, self.rank, self.world)
        assert self.vocab_local >= 1, "more ranks than vocabulary slices"
        self.device = torch.device(device)
        self.timeout_s = timeout_s
        rec = HEADER_BYTES + 8 * cand
        lay = RegionLayout()
        lay.add("flags", self.world * 4)
        lay.add("xchg", 2 * self.world * max_rows * rec)
        self.buf = SymmetricBuffer(lay.size, group, self.device)
        o = lay.offsets
        self.peer_xchg = torch.tensor([b + o["xchg"] for b in self.buf.peers], dtype=torch.int64, device=self.device)
        self.peer_flags = torch.tensor([b + o["flags"] for b in self.buf.peers], dtype=torch.int64,
                                       device=self.device)
        self.buf.view(o["flags"], (self.world,), torch.int32).zero_()
        self.seq = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.counter = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.inexact = torch.zeros(1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        barrier(group)

    @property
    def inexact_rows(self) -> int:
        """Rows drawn so far from an incomplete candidate union (host read, synchronizes)."""
        return int(self.inexact.item())

    def sample(self, logits_local: torch.Tensor, st: SamplingTensors | None = None, suppress=(-1, -1, -1),
               out: torch.Tensor | None = None, row_slot: torch.Tensor | None = None,
               slot_tokens: torch.Tensor | None = None, phases: int = 3) -> torch.Tensor:
        """logits_local: fp32 [rows, >= vocab_local] of this rank's slice (processed in place).
        Returns int32 tokens [rows], identical on every rank.  Same state semantics as
        ``ops.sample`` (``row_slot`` indexes the per-request state; ``seen`` is the
        full-vocabulary mask, updated with the drawn token on every rank)."""
        st = st or SamplingTensors()
        rows = logits_local.shape[0]
        if out is None:
            out = torch.empty(rows, dtype=torch.int32, device=logits_local.device)
        lo, hi, keep = suppress
        for a in range(0, max(rows, 1), self.max_rows):
            b = min(rows, a + self.max_rows)
            if b <= a:
                break
            rs = row_slot[a:b] if row_slot is not None else None
            if row_slot is None and a > 0:
                rs = torch.arange(a, b, dtype=torch.int32, device=logits_local.device)
            ext().vocab_sample(logits_local[a:b], out[a:b], self.peer_xchg, self.peer_flags, self.rank, self.world,
                               self.cand, self.max_rows, self.vocab0, self.vocab_local, self.vocab, self.seq,
                               self.counter, self.inexact, status_word(self.device), self.timeout_s,
                               st.temperature, st.top_k, st.top_p, st.min_p, st.rep_penalty, st.seen, lo, hi, keep,
                               st.seeds, st.step, rs, slot_tokens, phases)
        return out

    def close(self):
        self.buf.close()
