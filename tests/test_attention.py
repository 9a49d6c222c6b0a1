"""Paged prefill / decode and varlen attention kernels vs an fp32 oracle."""
import math

import pytest
import torch

from sglang_omni_b200.ops import attention as A


def _make_cache(kv_lens, hkv, d, device, seed=0):
    g = torch.Generator().manual_seed(seed)
    pages_needed = [(n + 63) // 64 for n in kv_lens]
    total = sum(pages_needed) + 3
    perm = torch.randperm(total, generator=g).tolist()
    k = (torch.randn(total, hkv, 64, d, generator=g) * 0.5).bfloat16()
    v = torch.randn(total, hkv, 64, d, generator=g).bfloat16()
    maxp = max(pages_needed)
    bt = torch.zeros(len(kv_lens), maxp, dtype=torch.int32)
    i = 0
    for b, n in enumerate(pages_needed):
        bt[b, :n] = torch.tensor(perm[i:i + n])
        i += n
    return k.to(device), v.to(device), bt.to(device)


def test_tile_rows_choice():
    assert A.prefill_tile_rows(128, 8) in (128, 256)
    assert A.prefill_tile_rows(128, 16) in (128, 256)
    assert A.prefill_tile_rows(64, 8) == 64


def test_prefill_tiles():
    req, tok0 = A.prefill_tiles([10, 0, 17], 8)
    assert req == [0, 0, 1 + 1, 2, 2] or req == [0, 0, 2, 2, 2]
    assert len(req) == len(tok0)


def test_paged_ref_matches_dense_sdpa():
    torch.manual_seed(0)
    kv_lens = [70]
    k, v, bt = _make_cache(kv_lens, 2, 16, "cpu")
    q = torch.randn(5, 4, 16)
    cu = torch.tensor([0, 5], dtype=torch.int32)
    out = A.paged_attention_ref(q, k, v, bt, cu, torch.tensor(kv_lens), 0.25, True)
    kk = A.gather_kv_ref(k, bt[0], 70).float().repeat_interleave(2, 1)
    vv = A.gather_kv_ref(v, bt[0], 70).float().repeat_interleave(2, 1)
    qq = q.permute(1, 0, 2)[None]
    mask = torch.ones(5, 70, dtype=torch.bool).tril(65)
    ref = torch.nn.functional.scaled_dot_product_attention(qq, kk.permute(1, 0, 2)[None], vv.permute(1, 0, 2)[None],
                                                           attn_mask=mask, scale=0.25)
    torch.testing.assert_close(out, ref[0].permute(1, 0, 2), atol=1e-4, rtol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [64, 128, 256])
@pytest.mark.parametrize("hq,hkv", [(32, 4), (16, 2), (32, 8), (16, 8)])
@pytest.mark.parametrize("q_lens,kv_extra", [([1, 7, 64, 130], [0, 5, 0, 100]), ([300], [0]), ([9, 1], [200, 1000])])
def test_prefill_paged(hq, hkv, q_lens, kv_extra, rows):
    """rows=64: the mma.sync kernel; rows=128: the tcgen05 kernel (TMEM S / O, TMA K/V pages);
    rows=256: its two-tile ping-pong variant."""
    _prefill_case(hq, hkv, q_lens, kv_extra, rows)


def _prefill_case(hq, hkv, q_lens, kv_extra, rows, q_scale=0.5, seed=0):
    d = 128
    kv_lens = [q + e for q, e in zip(q_lens, kv_extra)]
    k, v, bt = _make_cache(kv_lens, hkv, d, "cuda", seed=seed)
    T = sum(q_lens)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    q = (torch.randn(T, hq * d, device="cuda", generator=g) * q_scale).bfloat16()
    cu = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0).tolist()), dtype=torch.int32, device="cuda")
    kl = torch.tensor(kv_lens, dtype=torch.int32, device="cuda")
    req, tok0 = A.prefill_tiles(q_lens, hq // hkv, rows)
    tr = torch.tensor(req, dtype=torch.int32, device="cuda")
    tt = torch.tensor(tok0, dtype=torch.int32, device="cuda")
    out = A.prefill_attention(q, k, v, bt, cu, kl, tr, tt, hq, hkv, d, tile_rows=rows)
    torch.cuda.synchronize()
    from sglang_omni_b200.ops._ext import check_status

    check_status(torch.device("cuda", 0))
    ref = A.paged_attention_ref(q.view(T, hq, d), k, v, bt, cu, kl, 1 / math.sqrt(d), True)
    torch.testing.assert_close(out.float().view(T, hq, d), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("hq,hkv", [(16, 16), (32, 2), (32, 4)])
def test_prefill_tcgen05_long_and_rescaled(hq, hkv):
    """The tcgen05 kernel over many key blocks (1024-token prompts after a cached prefix), MHA and
    16-head groups, and large scores (q x 4) so the running max is raised and O rescaled in TMEM."""
    for rows in (128, 256):
        _prefill_case(hq, hkv, [1024, 333], [0, 700], rows, q_scale=0.5, seed=5)
        _prefill_case(hq, hkv, [512, 77], [64, 0], rows, q_scale=4.0, seed=6)


@pytest.mark.gpu
@pytest.mark.parametrize("hq,hkv,d", [(32, 4, 128), (16, 2, 128), (32, 8, 128), (16, 8, 128), (8, 8, 64)])
@pytest.mark.parametrize("kv_lens", [[1, 63, 64, 65, 1000], [3000, 17], [1100 + 7 * i for i in range(40)]])
def test_decode_paged(hq, hkv, d, kv_lens):
    k, v, bt = _make_cache(kv_lens, hkv, d, "cuda", seed=3)
    B = len(kv_lens)
    q = torch.randn(B, hq * d, device="cuda").bfloat16()
    kl = torch.tensor(kv_lens, dtype=torch.int32, device="cuda")
    ws = A.DecodeWorkspace(B, hq, d, max(kv_lens), "cuda", keys_per_split=256)
    out = A.decode_attention(q, k, v, bt, kl, hq, hkv, d, ws)
    cu = torch.arange(B + 1, dtype=torch.int32, device="cuda")
    ref = A.paged_attention_ref(q.view(B, hq, d), k, v, bt, cu, kl, 1 / math.sqrt(d), True)
    torch.testing.assert_close(out.float().view(B, hq, d), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.gpu
def test_decode_context_longer_than_workspace():
    """Contexts above max_splits * keys_per_split widen the split instead of overrunning the scratch."""
    kv_lens = [3000, 700, 5]
    hq, hkv, d = 16, 2, 128
    k, v, bt = _make_cache(kv_lens, hkv, d, "cuda", seed=5)
    B = len(kv_lens)
    q = torch.randn(B, hq * d, device="cuda").bfloat16()
    kl = torch.tensor(kv_lens, dtype=torch.int32, device="cuda")
    ws = A.DecodeWorkspace(B, hq, d, 512, "cuda", keys_per_split=256)  # 2 splits
    out = A.decode_attention(q, k, v, bt, kl, hq, hkv, d, ws)
    cu = torch.arange(B + 1, dtype=torch.int32, device="cuda")
    ref = A.paged_attention_ref(q.view(B, hq, d), k, v, bt, cu, kl, 1 / math.sqrt(d), True)
    torch.testing.assert_close(out.float().view(B, hq, d), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("h,d", [(20, 64), (16, 80), (16, 96), (16, 128)])
def test_varlen_noncausal(h, d):
    lens = [5, 100, 33, 200]
    T = sum(lens)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    qkv = (torch.randn(T, 3, h, d, device="cuda") * 0.5).bfloat16()
    q, k, v = qkv[:, 0].reshape(T, h * d), qkv[:, 1].reshape(T, h * d), qkv[:, 2].reshape(T, h * d)
    out = A.varlen_attention(q.contiguous(), k.contiguous(), v.contiguous(), cu, h, h, d)
    ref = A.varlen_attention_ref(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu, 1 / math.sqrt(d), False)
    torch.testing.assert_close(out.float().view(T, h, d), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [128, 256])
@pytest.mark.parametrize("h,hkv,d,causal", [(16, 16, 80, False), (16, 16, 128, False), (32, 4, 128, True),
                                             (16, 2, 96, True)])
def test_varlen_tcgen05_strided_views(rows, h, hkv, d, causal):
    """The tcgen05 kernels over ragged contiguous K/V: q / k / v are strided views of fused QKV
    rows (head dims below 128 load zeros past the head), long and short sequences, GQA groups."""
    import os

    lens = [5, 100, 333, 64, 700]
    T = sum(lens)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    width = (h + 2 * hkv) * d
    qkv = (torch.randn(T, width, device="cuda") * 0.5).bfloat16()
    q, k, v = qkv[:, :h * d], qkv[:, h * d:(h + hkv) * d], qkv[:, (h + hkv) * d:]
    old = os.environ.get("OMNI_FA_TILE_ROWS")
    os.environ["OMNI_FA_TILE_ROWS"] = str(rows)
    try:
        assert A.varlen_tile_rows(q, k, d, h // hkv, 0, v) == rows
        out = A.varlen_attention(q, k, v, cu, h, hkv, d, causal=causal, q_lens=lens)
    finally:
        if old is None:
            os.environ.pop("OMNI_FA_TILE_ROWS")
        else:
            os.environ["OMNI_FA_TILE_ROWS"] = old
    torch.cuda.synchronize()
    from sglang_omni_b200.ops._ext import check_status

    check_status(torch.device("cuda", 0))
    ref = A.varlen_attention_ref(q.reshape(T, h, d), k.reshape(T, hkv, d), v.reshape(T, hkv, d), cu,
                                 1 / math.sqrt(d), causal)
    torch.testing.assert_close(out.float().view(T, h, d), ref, atol=2e-2, rtol=2e-2)
