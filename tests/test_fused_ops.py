"""QK-norm + M-RoPE + KV store, MoE routing/combine, embedding and sampling kernels vs fp32 oracles."""
import pytest
import torch

from sglang_omni_b200.ops import embedding as Emb
from sglang_omni_b200.ops import moe as M
from sglang_omni_b200.ops import rope as R
from sglang_omni_b200.ops import sampling as S


def test_rope_ref_plain_matches_rotate_half():
    cos, sin = R.rope_tables(16, 10000.0, 64, round_bf16=False)
    x = torch.randn(5, 2, 16)
    pos = torch.arange(5, dtype=torch.int32)
    y = R.apply_rope_ref(x, pos, cos, sin, 16, True)
    c = torch.cat([cos[:5], cos[:5]], -1)[:, None]
    s = torch.cat([sin[:5], sin[:5]], -1)[:, None]
    rot = torch.cat([-x[..., 8:], x[..., :8]], -1)
    torch.testing.assert_close(y, x * c + rot * s)


def test_route_ref_topk():
    logits = torch.randn(4, 16)
    ids, w = M.route_ref(logits, 3)
    torch.testing.assert_close(w.sum(-1), torch.ones(4))
    assert (ids == logits.topk(3).indices).all()


@pytest.mark.gpu
@pytest.mark.parametrize("mrope", [False, True])
@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("d", [128, 32, 96])
def test_qkv_rope_store(mrope, neox, d):
    torch.manual_seed(0)
    T, hq, hkv = 37, 32, 4
    qkv = torch.randn(T, (hq + 2 * hkv) * d, device="cuda").bfloat16()
    qn = (1 + 0.1 * torch.randn(d, device="cuda")).bfloat16()
    kn = (1 + 0.1 * torch.randn(d, device="cuda")).bfloat16()
    cos, sin = R.rope_tables(d, 1e6, 4096, "cuda")
    if mrope:
        pos = torch.randint(0, 4000, (3, T), dtype=torch.int32, device="cuda")
        sec = [24, 20, 20] if d == 128 else [d // 2 - 2 * (d // 8), d // 8, d // 8]
    else:
        pos = torch.randint(0, 4000, (T,), dtype=torch.int32, device="cuda")
        sec = None
    pages = 2
    kc = torch.zeros(pages, hkv, 64, d, device="cuda").bfloat16()
    vc = torch.zeros_like(kc)
    slots = torch.randperm(pages * 64, device="cuda")[:T].to(torch.int32)
    slots[3] = -1
    a = qkv.clone()
    R.qkv_rope_store(a, hq, hkv, d, pos, cos, sin, q_norm=qn, k_norm=kn, neox=neox, mrope_section=sec,
                     slot_mapping=slots, k_cache=kc, v_cache=vc)
    b = qkv.clone()
    kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
    R.qkv_rope_store_ref(b, hq, hkv, d, qn, kn, 1e-6, pos, cos, sin, d, neox, sec, True, slots, kc2, vc2)
    torch.testing.assert_close(a.float(), b.float(), atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(kc.float(), kc2.float(), atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(vc.float(), vc2.float())


@pytest.mark.gpu
@pytest.mark.parametrize("T,E,k", [(1, 128, 8), (64, 128, 8), (333, 128, 6), (50, 64, 4)])
def test_fused_moe(T, E, k):
    torch.manual_seed(T + E)
    H, I = 256, 128
    x = torch.randn(T, H, device="cuda").bfloat16()
    wr = (torch.randn(E, H, device="cuda") * 0.1).bfloat16()
    w13 = (torch.randn(E, 2 * I, H, device="cuda") * 0.05).bfloat16()
    w2 = (torch.randn(E, H, I, device="cuda") * 0.05).bfloat16()
    ws = M.MoEWorkspace(T, E, k, H, I, "cuda")
    y = M.fused_moe(x, wr, w13, w2, k, ws)
    ref = M.moe_ref(x, wr, w13, w2, k)
    scale = ref.abs().max()
    assert ((y.float() - ref).abs().max() / scale) < 3e-2
    # offsets are a valid exclusive scan of the histogram
    off = ws.offsets.cpu()
    assert int(off[-1]) == T * k and (off[1:] >= off[:-1]).all()


@pytest.mark.gpu
def test_moe_shared_expert_combine():
    torch.manual_seed(5)
    T, E, k, H, I = 20, 32, 4, 128, 64
    x = torch.randn(T, H, device="cuda").bfloat16()
    wr = (torch.randn(E, H, device="cuda") * 0.1).bfloat16()
    w13 = (torch.randn(E, 2 * I, H, device="cuda") * 0.05).bfloat16()
    w2 = (torch.randn(E, H, I, device="cuda") * 0.05).bfloat16()
    shared = torch.randn(T, H, device="cuda").bfloat16()
    gate = torch.randn(T, 1, device="cuda")
    ws = M.MoEWorkspace(T, E, k, H, I, "cuda")
    y = M.fused_moe(x, wr, w13, w2, k, ws, shared_out=shared, shared_gate=gate)
    ref = M.moe_ref(x, wr, w13, w2, k) + torch.sigmoid(gate) * shared.float()
    assert ((y.float() - ref).abs().max() / ref.abs().max()) < 3e-2


@pytest.mark.gpu
def test_moe_routing_scratch_reused_across_calls():
    """The scatter re-zeroes its own histogram: back-to-back calls of different sizes on
    one workspace must each see fresh counts (no memset between them)."""
    E, k, H, I = 64, 4, 128, 64
    g = torch.Generator(device="cuda").manual_seed(3)
    wr = (torch.randn(E, H, device="cuda", generator=g) * 0.1).bfloat16()
    w13 = (torch.randn(E, 2 * I, H, device="cuda", generator=g) * 0.05).bfloat16()
    w2 = (torch.randn(E, H, I, device="cuda", generator=g) * 0.05).bfloat16()
    ws = M.MoEWorkspace(96, E, k, H, I, "cuda")
    for T in (96, 3, 57, 96, 1):
        x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
        y = M.fused_moe(x, wr, w13, w2, k, ws)
        ref = M.moe_ref(x, wr, w13, w2, k)
        assert ((y.float() - ref).abs().max() / ref.abs().max()) < 3e-2, T
        assert int(ws.offsets[E]) == T * k
        assert int(ws.counts.abs().sum()) == 0 and int(ws.cursor.abs().sum()) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("H,shared", [(2048, False), (4096, True), (1024, False)])
def test_moe_combine_fused_add_rmsnorm(H, shared):
    """combine + residual add + RMSNorm in one launch == unfused combine, then rms_norm(residual=...)."""
    from sglang_omni_b200.ops import norm as N

    torch.manual_seed(H)
    T, E, k, I = 33, 32, 8, 64
    x = torch.randn(T, H, device="cuda").bfloat16()
    wr = (torch.randn(E, H, device="cuda") * 0.05).bfloat16()
    w13 = (torch.randn(E, 2 * I, H, device="cuda") * 0.05).bfloat16()
    w2 = (torch.randn(E, H, I, device="cuda") * 0.05).bfloat16()
    so = torch.randn(T, H, device="cuda").bfloat16() if shared else None
    sg = torch.randn(T, 1, device="cuda") if shared else None
    nw = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16()
    res0 = torch.randn(T, H, device="cuda").bfloat16()
    ws = M.MoEWorkspace(T, E, k, H, I, "cuda")
    h = M.fused_moe(x, wr, w13, w2, k, ws, shared_out=so, shared_gate=sg)
    res_a = res0.clone()
    want = N.rms_norm(h, nw, 1e-6, residual=res_a)
    res_b = res0.clone()
    got = M.fused_moe(x, wr, w13, w2, k, ws, shared_out=so, shared_gate=sg, norm=(res_b, nw, 1e-6))
    torch.testing.assert_close(res_b, res_a, atol=0, rtol=0)
    torch.testing.assert_close(got, want, atol=1e-2, rtol=1e-2)
    # and against fp32
    r32 = res0.float() + h.float()
    ref = N.rms_norm_ref(r32, nw.float(), 1e-6)
    assert float((got.float() - ref).abs().max()) < 0.05


@pytest.mark.gpu
def test_group_limited_sigmoid_routing():
    torch.manual_seed(7)
    T, E = 40, 256
    logits = torch.randn(T, E, device="cuda")
    bias = torch.randn(E, device="cuda") * 0.1
    ids, w = M.route(logits, 8, mode=1, bias=bias, n_group=8, topk_group=4, renormalize=True, scaling=2.5)
    rid, rw = M.route_ref(logits, 8, 1, bias, 8, 4, True, 2.5)
    assert torch.equal(ids.sort(-1).values.cpu(), rid.sort(-1).values.cpu())
    torch.testing.assert_close(w.sort(-1).values, rw.sort(-1).values, atol=1e-5, rtol=1e-4)


@pytest.mark.gpu
def test_embed_mm_overwrite():
    table = torch.randn(1000, 256, device="cuda").bfloat16()
    ids = torch.randint(0, 1000, (50,), dtype=torch.int32, device="cuda")
    mm = torch.randn(7, 256, device="cuda").bfloat16()
    idx = torch.full((50,), -1, dtype=torch.int32, device="cuda")
    idx[10:17] = torch.arange(7, dtype=torch.int32, device="cuda")
    y = Emb.embed(ids, table, idx, mm)
    ref = Emb.embed(ids.cpu(), table.cpu(), idx.cpu(), mm.cpu())
    torch.testing.assert_close(y.cpu(), ref)


@pytest.mark.gpu
def test_sampling_greedy_and_penalty():
    torch.manual_seed(0)
    B, V = 6, 151936
    logits = torch.randn(B, V, device="cuda")
    st = S.SamplingTensors(temperature=torch.zeros(B, device="cuda"))
    tok = S.sample(logits.clone(), st)
    assert torch.equal(tok.long().cpu(), logits.argmax(-1).cpu())
    seen = torch.zeros(B, V, dtype=torch.uint8, device="cuda")
    seen[torch.arange(B), logits.argmax(-1)] = 1
    st = S.SamplingTensors(temperature=torch.zeros(B, device="cuda"), rep_penalty=torch.full((B,), 1e9, device="cuda"),
                           seen=seen)
    tok2 = S.sample(logits.clone(), st)
    ref = S.sample_ref(logits.cpu(), S.SamplingTensors(temperature=torch.zeros(B), rep_penalty=torch.full((B,), 1e9),
                                                        seen=torch.zeros(B, V, dtype=torch.uint8).index_put_(
                                                            (torch.arange(B), logits.argmax(-1).cpu()),
                                                            torch.ones(B, dtype=torch.uint8))))
    assert torch.equal(tok2.cpu(), ref)


@pytest.mark.gpu
def test_sampling_topk_topp_distribution():
    torch.manual_seed(1)
    V, N = 64, 4000
    base = torch.randn(V, device="cuda") * 2
    logits = base[None].repeat(N, 1)
    st = S.SamplingTensors(temperature=torch.full((N,), 0.8, device="cuda"),
                           top_k=torch.full((N,), 10, dtype=torch.int32, device="cuda"),
                           top_p=torch.full((N,), 0.9, device="cuda"),
                           seeds=torch.arange(N, dtype=torch.int64, device="cuda"),
                           step=torch.zeros(N, dtype=torch.int32, device="cuda"))
    tok = S.sample(logits.clone(), st).cpu().long()
    # expected distribution: top-k 10, then nucleus 0.9, renormalised
    x = base.cpu() / 0.8
    top = x.topk(10)
    p = torch.softmax(top.values, -1)
    cum = p.cumsum(0)
    keep = (cum - p) < 0.9
    pk = torch.where(keep, p, torch.zeros_like(p))
    pk /= pk.sum()
    emp = torch.bincount(tok, minlength=V).float() / N
    exp = torch.zeros(V)
    exp[top.indices] = pk
    assert (emp - exp).abs().max() < 0.04
    assert emp[exp == 0].sum() < 0.01


@pytest.mark.gpu
def test_sampling_topp_large_vocab_candidates():
    """Top-p alone over a 151936-token row whose mass sits on 100 tokens: the candidates fit in
    shared memory; the draws follow the renormalised nucleus."""
    torch.manual_seed(2)
    V, N, K = 151936, 1500, 100
    base = torch.full((V,), -60.0)
    hot = torch.randperm(V)[:K]
    base[hot] = torch.randn(K) * 1.5
    logits = base.cuda()[None].repeat(N, 1)
    st = S.SamplingTensors(temperature=torch.ones(N, device="cuda"), top_p=torch.full((N,), 0.9, device="cuda"),
                           seeds=torch.arange(N, dtype=torch.int64, device="cuda"),
                           step=torch.zeros(N, dtype=torch.int32, device="cuda"))
    tok = S.sample(logits, st).cpu().long()
    p = torch.softmax(base.double(), -1)
    ps, order = p.sort(descending=True)
    keep = (ps.cumsum(0) - ps) < 0.9
    exp = torch.zeros(V, dtype=torch.float64)
    exp[order[keep]] = ps[keep] / ps[keep].sum()
    emp = torch.bincount(tok, minlength=V).double() / N
    assert emp[exp == 0].sum() == 0
    assert (emp - exp).abs().max() < 0.05


@pytest.mark.gpu
def test_sampling_topp_flat_row_full_sweep():
    """A flat 20000-token row leaves more candidates than shared memory holds: top-p and the
    draw sweep the row; every draw must lie in the nucleus."""
    torch.manual_seed(3)
    V, N = 20000, 256
    base = torch.randn(V) * 0.3
    logits = base.cuda()[None].repeat(N, 1)
    st = S.SamplingTensors(temperature=torch.ones(N, device="cuda"), top_p=torch.full((N,), 0.5, device="cuda"),
                           seeds=torch.arange(N, dtype=torch.int64, device="cuda"),
                           step=torch.zeros(N, dtype=torch.int32, device="cuda"))
    tok = S.sample(logits, st).cpu().long()
    p = torch.softmax(base.double(), -1)
    ps, order = p.sort(descending=True)
    keep = (ps.cumsum(0) - ps) < 0.5 + 1e-3     # bisection tolerance at the boundary
    allowed = torch.zeros(V, dtype=torch.bool)
    allowed[order[keep]] = True
    assert bool(allowed[tok].all())
    assert len(set(tok.tolist())) > N // 3      # draws spread over the nucleus


@pytest.mark.gpu
def test_rope_half_inplace_matches_fp32_reference():
    """The vision tower's in-place 2-D RoPE on padded q / k heads of fused QKV rows: rotated
    columns match the fp32 rotate-half formula, padding columns and v stay untouched."""
    from sglang_omni_b200.ops.rope import rope_half_inplace

    T, nh, kd, hd = 300, 16, 80, 72
    g = torch.Generator().manual_seed(3)
    qkv = torch.randn(T, 3 * nh * kd, generator=g).bfloat16()
    qkv.view(T, 3, nh, kd)[..., hd:] = 0
    ang = torch.rand(T, hd // 2, generator=g) * 20
    ang = torch.cat([ang, ang], -1)
    cos, sin = ang.cos(), ang.sin()
    ref = rope_half_inplace(qkv.clone(), 2 * nh, kd, hd, cos, sin)          # CPU: the torch formula
    got = rope_half_inplace(qkv.cuda(), 2 * nh, kd, hd, cos.cuda(), sin.cuda()).cpu()
    torch.testing.assert_close(got.float(), ref.float(), atol=1e-2, rtol=1e-2)
    assert torch.equal(got.view(T, 3, nh, kd)[:, 2], qkv.view(T, 3, nh, kd)[:, 2])
    assert not got.view(T, 3, nh, kd)[..., hd:].any()
