"""Bounded device waits that run out (one GPU, no fault).

Every cross-rank wait inside a kernel polls a flag with a wall-clock limit. Here
each kind of wait is given a flag that nothing will ever set and a 10 ms limit:
the kernel must give up, record status 2 (peer timeout) in the device status
word, and return, so that the context stays usable: the next kernel on the same
stream runs and computes the right result, and ``check_status`` raises on the
host.  The waits covered are the EP w13 GEMM's wait for the dispatch flags
(before it reads the expert counts), the MoE combine's wait for the owners'
flags, and the dense GEMM's wait for an all-gather before its first operand
load (the tensor-parallel consumer GEMM).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

LIMIT_S = 0.01


def _status_then_recover(dev):
    from sglang_omni_b200.ops import gemm
    from sglang_omni_b200.ops._ext import check_status, status_word

    torch.cuda.synchronize(dev)
    assert int(status_word(dev).item()) == 2, "the wait should have timed out with status 2"
    # the context is still usable: a plain GEMM right after computes the right thing
    x = torch.randn(32, 256, device=dev).bfloat16()
    w = (torch.randn(128, 256, device=dev) * 0.05).bfloat16()
    y = gemm.linear(x, w)
    torch.testing.assert_close(y.float(), gemm.linear_ref(x.cpu(), w.cpu()).float().to(dev), atol=2e-2, rtol=2e-2)
    with pytest.raises(RuntimeError, match="peer flag wait timed out"):
        check_status(dev)
    check_status(dev)  # cleared by the raise


def test_ep_gemm_setup_wait_times_out():
    from sglang_omni_b200.ops._ext import ext, status_word

    dev = torch.device("cuda", 0)
    status_word(dev).zero_()
    G, cap, H, I = 4, 32, 256, 128
    w13 = (torch.randn(G, 2 * I, H, device=dev) * 0.05).bfloat16()
    x = torch.randn(G * cap, H, device=dev).bfloat16()
    h = torch.zeros(G * cap, I, device=dev).bfloat16()
    counts = torch.full((G,), 5, dtype=torch.int32, device=dev)
    copy = torch.full((G,), -1, dtype=torch.int32, device=dev)
    flags = torch.zeros(2, dtype=torch.int32, device=dev)     # nobody ever raises these
    seq = torch.full((1,), 7, dtype=torch.int32, device=dev)
    ext().gemm_ep(w13, x, h, I, True, cap, counts, copy, flags, seq, LIMIT_S, None, None, 0, None, None, None,
                  None, 5, status_word(dev))
    torch.cuda.synchronize(dev)
    # after the timeout the groups are taken as empty: nothing computed, counts copied as 0
    assert copy.tolist() == [0] * G
    assert int(h.abs().sum()) == 0
    _status_then_recover(dev)


def test_moe_combine_wait_times_out():
    from sglang_omni_b200.ops._ext import ext, status_word

    dev = torch.device("cuda", 0)
    status_word(dev).zero_()
    T, k, H = 8, 4, 256
    y = torch.randn(T * k, H, device=dev).bfloat16()
    inv = torch.arange(T * k, dtype=torch.int32, device=dev).view(T, k)
    w = torch.full((T, k), 0.25, device=dev)
    out = torch.empty(T, H, device=dev).bfloat16()
    flags = torch.zeros(3, dtype=torch.int32, device=dev)
    seq = torch.full((1,), 1, dtype=torch.int32, device=dev)
    ext().moe_combine(y, inv, w, out, wait_flags=flags, wait_seq=seq, status=status_word(dev), timeout_s=LIMIT_S)
    torch.cuda.synchronize(dev)
    ref = (y.float().view(T, k, H) * 0.25).sum(1)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)   # it still ran after giving up
    _status_then_recover(dev)


def test_gemm_gather_wait_times_out():
    from sglang_omni_b200.ops import gemm
    from sglang_omni_b200.ops._ext import status_word

    dev = torch.device("cuda", 0)
    status_word(dev).zero_()
    x = torch.randn(64, 512, device=dev).bfloat16()
    w = (torch.randn(256, 512, device=dev) * 0.05).bfloat16()
    flags = torch.zeros(2, dtype=torch.int32, device=dev)
    seq = torch.full((1,), 3, dtype=torch.int32, device=dev)
    y = gemm.linear(x, w, wait=(flags, seq, LIMIT_S))
    torch.cuda.synchronize(dev)
    torch.testing.assert_close(y.float(), gemm.linear_ref(x.cpu(), w.cpu()).float().to(dev), atol=2e-2, rtol=2e-2)
    _status_then_recover(dev)
