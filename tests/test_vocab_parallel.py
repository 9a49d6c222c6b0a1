"""Vocab-parallel sampling (csrc/vocab_parallel.cu, parallel/vocab.py).

The multi-rank exchange is emulated on one GPU: every emulated rank has its own
exchange region, flags and sequence number, the local phase of every rank runs
first (each stores its records into every rank's region and sets the flags),
then the merge of every rank -- no kernel waits for another one that has not
already finished.  Every rank's tokens must equal the single-GPU fused sampler's
for the rules the design makes exact, with no row counted as inexact.
"""
import socket

import pytest
import torch

from sglang_omni_b200.ops.sampling import SamplingTensors, sample
from sglang_omni_b200.parallel.vocab import HEADER_BYTES, vocab_slice

gpu = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")


def test_vocab_slice_cover():
    for V in (151936, 1000, 4099):
        for w in (1, 2, 3, 4, 8):
            got = [vocab_slice(V, r, w) for r in range(w)]
            assert all(g[2] % 16 == 0 for g in got)
            assert sum(g[1] for g in got) == V
            assert all(got[r][0] == (got[r - 1][0] + got[r - 1][1]) for r in range(1, w))


def _state(rows, V, dev, temp, top_k=0, top_p=1.0, min_p=0.0, rep=1.0):
    g = torch.Generator(device="cpu").manual_seed(3)
    return SamplingTensors(
        temperature=torch.full((rows,), temp, device=dev),
        top_k=torch.full((rows,), top_k, dtype=torch.int32, device=dev),
        top_p=torch.full((rows,), top_p, device=dev),
        min_p=torch.full((rows,), min_p, device=dev),
        rep_penalty=torch.full((rows,), rep, device=dev),
        seen=(torch.rand(rows, V, generator=g) < 0.01).to(torch.uint8).to(dev),
        seeds=torch.arange(rows, dtype=torch.int64, device=dev) * 7919 + 11,
        step=torch.full((rows,), 5, dtype=torch.int32, device=dev))


def _clone(st):
    return SamplingTensors(*[None if t is None else t.clone() for t in (
        st.temperature, st.top_k, st.top_p, st.min_p, st.rep_penalty, st.seen, st.seeds, st.step)])


def _emulated(logits, st, world, cand, suppress=(-1, -1, -1)):
    """Tokens of every emulated rank + the inexact counters."""
    from sglang_omni_b200.ops._ext import ext, status_word

    dev = logits.device
    rows, V = logits.shape
    rec = HEADER_BYTES + 8 * cand
    max_rows = rows
    xchg = [torch.zeros(2 * world * max_rows * rec, dtype=torch.uint8, device=dev) for _ in range(world)]
    flags = [torch.zeros(world, dtype=torch.int32, device=dev) for _ in range(world)]
    peer_x = torch.tensor([t.data_ptr() for t in xchg], dtype=torch.int64, device=dev)
    peer_f = torch.tensor([t.data_ptr() for t in flags], dtype=torch.int64, device=dev)
    seqs = [torch.zeros(1, dtype=torch.int32, device=dev) for _ in range(world)]
    ctrs = [torch.zeros(1, dtype=torch.int32, device=dev) for _ in range(world)]
    inex = [torch.zeros(1, dtype=torch.int32, device=dev) for _ in range(world)]
    sts = [_clone(st) for _ in range(world)]
    outs = [torch.full((rows,), -1, dtype=torch.int32, device=dev) for _ in range(world)]
    slices = [vocab_slice(V, r, world) for r in range(world)]
    locs = []
    for r, (v0, vl, width) in enumerate(slices):
        loc = torch.full((rows, width), float("-inf"), device=dev)
        loc[:, :vl] = logits[:, v0:v0 + vl]
        locs.append(loc)
    for phase in (1, 2):
        for r, (v0, vl, _) in enumerate(slices):
            s = sts[r]
            ext().vocab_sample(locs[r], outs[r], peer_x, peer_f, r, world, cand, max_rows, v0, vl, V, seqs[r],
                               ctrs[r], inex[r], status_word(dev), 1.0, s.temperature, s.top_k, s.top_p, s.min_p,
                               s.rep_penalty, s.seen, *suppress, s.seeds, s.step, None, None, phase)
    torch.cuda.synchronize()
    return outs, [int(i.item()) for i in inex], sts


CASES = [
    dict(temp=0.0),
    dict(temp=0.8),
    dict(temp=0.7, top_k=20),
    dict(temp=1.0, top_k=50, top_p=0.8, min_p=0.02),
    dict(temp=0.6, top_p=0.9, peaked=True),
    dict(temp=0.9, min_p=0.1, peaked=True),
    dict(temp=0.0, rep=1.3, suppress=(1000, 2000, 1500)),
    dict(temp=1.0, top_k=64, rep=1.2, suppress=(0, 100, 7)),
]


@gpu
@needs_cuda
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_emulated_ranks_match_full_sampler(world, case):
    c = dict(CASES[case])
    dev = torch.device("cuda", 0)
    rows, V = 24, 151936
    g = torch.Generator(device=dev).manual_seed(100 + case)
    logits = torch.randn(rows, V, device=dev, generator=g) * (6.0 if c.pop("peaked", False) else 2.0)
    suppress = c.pop("suppress", (-1, -1, -1))
    st = _state(rows, V, dev, **c)
    st_full = _clone(st)
    ref = sample(logits.clone(), st_full, suppress)
    outs, inexact, sts = _emulated(logits, st, world, 64, suppress)
    for r in range(world):
        assert torch.equal(outs[r], ref), f"rank {r}: {outs[r].tolist()} vs {ref.tolist()}"
        assert inexact[r] == 0
        assert torch.equal(sts[r].step, st_full.step)
        assert torch.equal(sts[r].seen, st_full.seen)


@gpu
@needs_cuda
def test_flat_top_p_counts_inexact_rows():
    """A flat distribution with top-p only keeps far more tokens than the candidate union:
    the rows are still drawn (a valid token of the union) and counted as inexact."""
    dev = torch.device("cuda", 0)
    rows, V, world = 8, 151936, 4
    logits = torch.randn(rows, V, device=dev, generator=torch.Generator(device=dev).manual_seed(1)) * 0.1
    st = _state(rows, V, dev, temp=1.0, top_p=0.95)
    outs, inexact, _ = _emulated(logits, st, world, 64)
    assert all(i == rows for i in inexact)
    for r in range(1, world):
        assert torch.equal(outs[r], outs[0])
    assert int(outs[0].min()) >= 0 and int(outs[0].max()) < V


@gpu
@needs_cuda
def test_sampler_world1_loopback():
    """The sampler class over a one-rank group (its peer table is this GPU only)."""
    from sglang_omni_b200.parallel.hostgroup import HostGroup
    from sglang_omni_b200.parallel.vocab import VocabParallelSampler

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dev = torch.device("cuda", 0)
    vs = VocabParallelSampler(5000, 16, dev, group=HostGroup("127.0.0.1", port, 0, 1), cand=32)
    try:
        g = torch.Generator(device=dev).manual_seed(2)
        for step in range(3):   # consecutive exchanges alternate the record halves
            logits = torch.randn(20, 5000, device=dev, generator=g) * 3   # 20 rows > max_rows: two chunks
            st = _state(20, 5000, dev, temp=0.7, top_k=16)
            st2 = _clone(st)
            ref = sample(logits.clone(), st2)
            got = vs.sample(logits.clone(), st)
            torch.cuda.synchronize()
            assert torch.equal(got, ref)
        assert vs.inexact_rows == 0
    finally:
        vs.close()
