"""tcgen05 GEMM (csrc/gemm_sm100.cu) against an fp32 PyTorch oracle."""
import pytest
import torch

from sglang_omni_b200.ops import gemm as L


def _close(out, ref, tol=2e-2):
    out = out.float()
    ref = ref.float()
    scale = ref.abs().max().clamp_min(1.0)
    err = (out - ref).abs().max() / scale
    assert err < tol, f"max rel err {err.item():.4g}"


def test_linear_cpu_matches_ref():
    torch.manual_seed(0)
    x = torch.randn(5, 64)
    w = torch.randn(32, 64)
    y = L.linear(x, w)
    torch.testing.assert_close(y, x @ w.t())


def test_grouped_cpu_ref():
    torch.manual_seed(0)
    x = torch.randn(10, 16)
    w = torch.randn(3, 8, 16)
    off = torch.tensor([0, 4, 4, 10], dtype=torch.int32)
    y = L.grouped_linear(x, w, off)
    torch.testing.assert_close(y[:4], x[:4] @ w[0].t())
    torch.testing.assert_close(y[4:], x[4:] @ w[2].t())


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [1, 7, 16, 33, 100, 300, 1000])
@pytest.mark.parametrize("n,k", [(128, 64), (256, 2048), (1152, 200), (200, 128), (384, 4304)])
def test_dense_linear(rows, n, k):
    torch.manual_seed(rows * 7 + n)
    x = (torch.randn(rows, k, device="cuda") * 0.5).bfloat16()
    w = (torch.randn(n, k, device="cuda") * 0.05).bfloat16()
    y = L.linear(x, w)
    torch.cuda.synchronize()
    _close(y, L.linear_ref(x, w, out_dtype=torch.float32))


@pytest.mark.gpu
@pytest.mark.parametrize("act", [None, "gelu_tanh", "gelu", "silu"])
def test_linear_bias_act_residual(act):
    torch.manual_seed(1)
    rows, n, k = 77, 384, 256
    x = torch.randn(rows, k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") * 0.05).bfloat16()
    b = torch.randn(n, device="cuda").bfloat16()
    r = torch.randn(rows, n, device="cuda").bfloat16()
    y = L.linear(x, w, bias=b, residual=r, act=act)
    _close(y, L.linear_ref(x, w, b, r, act, torch.float32))


@pytest.mark.gpu
def test_linear_fp32_out():
    torch.manual_seed(2)
    x = torch.randn(64, 2048, device="cuda").bfloat16()
    w = (torch.randn(1024, 2048, device="cuda") * 0.02).bfloat16()
    y = L.linear(x, w, out_dtype=torch.float32)
    assert y.dtype == torch.float32
    _close(y, L.linear_ref(x, w, out_dtype=torch.float32), 1e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("groups,avg", [(8, 3), (16, 40), (128, 4), (4, 300)])
def test_grouped(gated, groups, avg):
    torch.manual_seed(groups + avg)
    counts = torch.randint(0, 2 * avg + 1, (groups,))
    counts[0] = 0
    offs = torch.zeros(groups + 1, dtype=torch.int32)
    offs[1:] = counts.cumsum(0)
    rows = int(offs[-1])
    k, n = 256, 256
    x = torch.randn(max(rows, 1), k, device="cuda").bfloat16()[:rows]
    w = (torch.randn(groups, 2 * n if gated else n, k, device="cuda") * 0.05).bfloat16()
    offs_d = offs.cuda()
    y = L.grouped_linear(x, w, offs_d, gated=gated, expected_rows=avg)
    ref = L.grouped_linear_ref(x, w, offs_d, gated, torch.float32)
    _close(y, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("rows,n,k", [(64, 5120, 2048), (64, 128, 2048), (7, 2048, 4096), (200, 256, 1024)])
def test_splitk_dense_repeated(rows, n, k):
    """Small-tile GEMMs take the split-K path (partials + reduce kernel); back-to-back
    calls must agree (bias + residual applied in the reduction)."""
    torch.manual_seed(rows + n)
    x = torch.randn(rows, k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") * 0.02).bfloat16()
    b = torch.randn(n, device="cuda").bfloat16()
    r = torch.randn(rows, n, device="cuda").bfloat16()
    ref = L.linear_ref(x, w, b, r, None, torch.float32)
    y1 = L.linear(x, w, bias=b, residual=r)
    y2 = L.linear(x, w, bias=b, residual=r)
    _close(y1, ref)
    _close(y2, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [1, 2, 3])
@pytest.mark.parametrize("rows,n,k,act,f32", [(64, 5120, 2048, None, False), (64, 130, 2048, "gelu", False),
                                              (16, 2048, 4096, "silu", False), (33, 128, 2048, None, True),
                                              (64, 516, 1024, "gelu_tanh", True)])
def test_splitk_finalisers(monkeypatch, mode, rows, n, k, act, f32):
    """Every split-K finaliser (second kernel / last split in the GEMM / cluster DSMEM reduce) against the fp32 oracle,
    with bias, activation and residual, bf16 and fp32 outputs, and output widths that are not a
    multiple of the 4-wide vector stores; two calls in a row must agree bit for bit."""
    monkeypatch.setattr(L, "_SPLITK_MODE", mode)
    torch.manual_seed(rows + n + mode)
    x = torch.randn(rows, k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") * 0.02).bfloat16()
    b = torch.randn(n, device="cuda").bfloat16()
    r = None if f32 else torch.randn(rows, n, device="cuda").bfloat16()
    dt = torch.float32 if f32 else None
    ref = L.linear_ref(x, w, b, r, act, torch.float32)
    y1 = L.linear(x, w, bias=b, residual=r, act=act, out_dtype=dt)
    y2 = L.linear(x, w, bias=b, residual=r, act=act, out_dtype=dt)
    _close(y1, ref, 1e-2 if f32 else 2e-2)
    assert torch.equal(y1, y2)


@pytest.mark.gpu
@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("rows,n,k", [(64, 1024, 2048), (16, 768, 1024), (300, 512, 512)])
def test_static_weight_prefetch(gated, rows, n, k):
    """Dense GEMMs inside static_weights() fetch their first weight tiles before the previous
    kernel finishes (programmatic dependent launch); gate and up halves, every shape path."""
    from sglang_omni_b200.ops import _ext

    torch.manual_seed(rows + n)
    x = torch.randn(rows, k, device="cuda").bfloat16()
    w = (torch.randn(2 * n if gated else n, k, device="cuda") * 0.05).bfloat16()
    ref = L.linear_ref(x, w, out_dtype=torch.float32, gated=gated)
    x2 = torch.empty_like(x)
    with L.static_weights():
        x2.copy_(x)                      # the activations come from the kernel right before
        y = L.linear(x2, w, gated=gated)
    torch.cuda.synchronize()
    _ext.check_status(x.device)
    _close(y, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("rows,n,k,f32", [(300, 512, 256, True), (1000, 1152, 512, False), (130, 264, 128, False)])
def test_wide_tile_staged_epilogue(rows, n, k, f32):
    """Token tiles of 128 / 256 stage the epilogue through shared memory (16-byte stores):
    fp32 and bf16 outputs, bias + residual, partial last token tiles and feature tiles."""
    torch.manual_seed(rows + n)
    x = torch.randn(rows, k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") * 0.05).bfloat16()
    b = torch.randn(n, device="cuda").bfloat16()
    r = None if f32 else torch.randn(rows, n, device="cuda").bfloat16()
    y = L.linear(x, w, bias=b, residual=r, out_dtype=torch.float32 if f32 else None)
    _close(y, L.linear_ref(x, w, b, r, None, torch.float32), 1e-2 if f32 else 2e-2)
