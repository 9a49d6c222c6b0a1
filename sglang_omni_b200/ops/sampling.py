"""Fused logits processing + sampling (csrc/fused_ops.cu ``sample_kernel``).

Per row: codec-range suppression, repetition penalty over a seen-token mask,
temperature, top-k (radix select), min-p, top-p (threshold search), then a
Gumbel-max draw from a counter-based hash (SplitMix64) keyed by (seed, step,
token).  Temperature 0 is greedy argmax (lowest index wins ties).

Reference counterparts: sglang_omni/engines/omni/runtime/sglang_ar.py:882-940
(suppress tokens, repetition penalty) and :1030 (model_runner.sample);
top_k_top_p_sampling_from_probs in sglang_omni/models/qwen3_omni/talker.py:926.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _check
from ._ext import ext


@dataclass
class SamplingTensors:
    temperature: torch.Tensor | None = None
    top_k: torch.Tensor | None = None
    top_p: torch.Tensor | None = None
    min_p: torch.Tensor | None = None
    rep_penalty: torch.Tensor | None = None
    seen: torch.Tensor | None = None
    seeds: torch.Tensor | None = None
    step: torch.Tensor | None = None


def process_logits_ref(logits, st: SamplingTensors, suppress=(-1, -1, -1)):
    x = logits.float().clone()
    lo, hi, keep = suppress
    if lo >= 0:
        mask = torch.zeros(x.shape[1], dtype=torch.bool, device=x.device)
        mask[lo:hi] = True
        if 0 <= keep < x.shape[1]:
            mask[keep] = False
        x[:, mask] = float("-inf")
    if st.rep_penalty is not None and st.seen is not None:
        rp = st.rep_penalty.float()[:, None]
        seen = st.seen.bool()
        pen = torch.where(x > 0, x / rp, x * rp)
        x = torch.where(seen, pen, x)
    if st.temperature is not None:
        t = st.temperature.float()[:, None]
        x = torch.where(t > 0, x / t.clamp_min(1e-30), x)
    return x


def sample_ref(logits, st: SamplingTensors, suppress=(-1, -1, -1), generator=None):
    x = process_logits_ref(logits, st, suppress)
    out = torch.empty(x.shape[0], dtype=torch.int32, device=x.device)
    for r in range(x.shape[0]):
        t = float(st.temperature[r]) if st.temperature is not None else 0.0
        row = x[r]
        if t <= 0:
            out[r] = int(torch.argmax(row))
            continue
        keep = torch.isfinite(row)
        if st.top_k is not None and 0 < int(st.top_k[r]) < row.numel():
            kth = row.topk(int(st.top_k[r])).values[-1]
            keep &= row >= kth
        if st.min_p is not None and float(st.min_p[r]) > 0:
            keep &= row >= row.max() + torch.log(st.min_p[r].float())
        probs = torch.softmax(row.masked_fill(~keep, float("-inf")), -1)
        if st.top_p is not None and float(st.top_p[r]) < 1:
            sp, si = probs.sort(descending=True)
            cum = sp.cumsum(0)
            cut = (cum - sp) >= float(st.top_p[r])
            sp[cut] = 0
            probs = torch.zeros_like(probs).scatter_(0, si, sp)
            probs = probs / probs.sum()
        out[r] = int(torch.multinomial(probs, 1, generator=generator))
    if st.seen is not None:
        st.seen[torch.arange(x.shape[0]), out.long()] = 1
    return out


def _gather_state(st: SamplingTensors, idx: torch.Tensor) -> SamplingTensors:
    g = lambda t: None if t is None else t[idx]  # noqa: E731
    return SamplingTensors(g(st.temperature), g(st.top_k), g(st.top_p), g(st.min_p), g(st.rep_penalty), g(st.seen),
                           g(st.seeds), g(st.step))


def sample(logits: torch.Tensor, st: SamplingTensors | None = None, suppress=(-1, -1, -1),
           out: torch.Tensor | None = None, row_slot: torch.Tensor | None = None,
           slot_tokens: torch.Tensor | None = None) -> torch.Tensor:
    """Returns int32 token ids [rows]. Modifies `logits` in place on the GPU path.

    With ``row_slot`` the per-request state arrays of ``st`` are indexed by
    slot (row r uses state row_slot[r]); the drawn token is also stored at
    ``slot_tokens[row_slot[r]]`` and the slot's step counter advances.
    """
    st = st or SamplingTensors()
    if not logits.is_cuda:
        if row_slot is not None:
            idx = row_slot.long()
            sub = _gather_state(st, idx)
            r = sample_ref(logits, sub, suppress)
            if st.seen is not None:
                st.seen[idx] = sub.seen
            if st.step is not None:
                st.step[idx] += 1
            if slot_tokens is not None:
                slot_tokens[idx] = r
        else:
            r = sample_ref(logits, st, suppress)
        if out is not None:
            out.copy_(r)
            return out
        return r
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    lo, hi, keep = suppress
    if _check.enabled() and row_slot is not None:
        arrs = [t for t in (st.temperature, st.top_k, st.seeds, st.step) if t is not None]
        if arrs:
            _check.check_range("sample", "row_slot", row_slot, 0, min(t.shape[0] for t in arrs))
        if slot_tokens is not None:
            _check.check_range("sample", "row_slot", row_slot, 0, slot_tokens.shape[0])
    ext().sample(logits, out, st.temperature, st.top_k, st.top_p, st.min_p, st.rep_penalty, st.seen, lo, hi, keep,
                 st.seeds, st.step, row_slot, slot_tokens)
    return out
