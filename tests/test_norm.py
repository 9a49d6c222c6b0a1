import pytest
import torch

from sglang_omni_b200.ops import norm as N


def test_rmsnorm_cpu_residual():
    x = torch.randn(4, 32)
    r = torch.randn(4, 32)
    r0 = r.clone()
    w = torch.randn(32)
    y = N.rms_norm(x, w, 1e-6, residual=r)
    torch.testing.assert_close(r, r0 + x)
    torch.testing.assert_close(y, N.rms_norm_ref(r0 + x, w, 1e-6))


@pytest.mark.gpu
@pytest.mark.parametrize("rows,h", [(1, 64), (17, 1024), (300, 2048), (5, 2560), (3, 128)])
def test_rmsnorm_gpu(rows, h):
    x = torch.randn(rows, h, device="cuda").bfloat16()
    w = torch.randn(h, device="cuda").bfloat16()
    y = N.rms_norm(x, w, 1e-6)
    ref = N.rms_norm_ref(x.float(), w.float(), 1e-6)
    torch.testing.assert_close(y.float(), ref, atol=3e-2, rtol=3e-2)


@pytest.mark.gpu
def test_fused_add_rmsnorm_gpu():
    x = torch.randn(33, 2048, device="cuda").bfloat16()
    r = torch.randn(33, 2048, device="cuda").bfloat16()
    w = torch.randn(2048, device="cuda").bfloat16()
    s = (x.float() + r.float()).bfloat16()
    y = N.rms_norm(x, w, 1e-6, residual=r)
    torch.testing.assert_close(r, s)
    torch.testing.assert_close(y.float(), N.rms_norm_ref(s.float(), w.float(), 1e-6), atol=3e-2, rtol=3e-2)


@pytest.mark.gpu
def test_layernorm_gpu():
    x = torch.randn(50, 1280, device="cuda").bfloat16()
    w = torch.randn(1280, device="cuda").bfloat16()
    b = torch.randn(1280, device="cuda").bfloat16()
    y = N.layer_norm(x, w, b, 1e-5)
    ref = torch.nn.functional.layer_norm(x.float(), (1280,), w.float(), b.float(), 1e-5)
    torch.testing.assert_close(y.float(), ref, atol=5e-2, rtol=3e-2)
