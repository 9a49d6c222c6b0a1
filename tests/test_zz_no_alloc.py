"""Allocation-free decode attention (C symbol omni_attention_decode_noalloc).

Callers that cannot allocate device memory (a stream capture owned by another
library, host runtimes that pass only inputs and outputs, custom allocators)
use this entry point; its split-KV scratch is a static device array inside the
library.  The test calls the exported C symbol through ctypes and compares its
output with the torch entry point's (which takes a caller-allocated
workspace) and with a plain fp32 PyTorch restatement of the attention, on two
calls in a row with different inputs, so a stale scratch from the first call
would show up in the second.  Both cases hold an empty-context row (a padding
row of a batch bucket), which must come back as zeros.  Arguments the kernel
cannot take are refused before anything is launched.  This file is collected
last on purpose.
"""
import ctypes
import math

import pytest
import torch


def _lib():
    import sglang_omni_b200._C as C  # loads libtorch / libc10 first

    lib = ctypes.CDLL(C.__file__)
    fn = lib.omni_attention_decode_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong,
                   ctypes.c_void_p]
    return fn


def _case(kv_lens, hq, hkv, d, seed):
    g = torch.Generator().manual_seed(seed)
    pages = [max(1, (n + 63) // 64) for n in kv_lens]
    total = sum(pages) + 1
    k = (torch.randn(total, hkv, 64, d, generator=g) * 0.5).bfloat16().cuda()
    v = torch.randn(total, hkv, 64, d, generator=g).bfloat16().cuda()
    perm = torch.randperm(total, generator=g).tolist()
    bt = torch.zeros(len(kv_lens), max(pages), dtype=torch.int32)
    i = 0
    for b, n in enumerate(pages):
        bt[b, :n] = torch.tensor(perm[i:i + n])
        i += n
    q = torch.randn(len(kv_lens), hq * d, generator=g).bfloat16().cuda()
    return q, k, v, bt.cuda(), torch.tensor(kv_lens, dtype=torch.int32).cuda()


def _call(fn, q, k, v, bt, kl, hq, hkv, d, kps, splits, num_pages=None):
    out = torch.full((q.shape[0], hq * d), float("nan"), dtype=torch.bfloat16, device="cuda")
    rc = fn(q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), bt.data_ptr(), bt.stride(0), kl.data_ptr(),
            q.shape[0], hq, hkv, d, 1.0 / math.sqrt(d), kps, splits,
            k.shape[0] if num_pages is None else num_pages, out.data_ptr(), out.stride(0),
            torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc, out


@pytest.mark.gpu
def test_noalloc_decode_matches_torch_entry():
    from sglang_omni_b200.ops import attention as A

    fn = _lib()
    hq, hkv, d = 32, 4, 128
    for call, (kv_lens, seed) in enumerate([([1, 700, 0, 64, 1500], 11), ([2000, 3, 129, 0], 12)]):
        q, k, v, bt, kl = _case(kv_lens, hq, hkv, d, seed)
        ws = A.DecodeWorkspace(len(kv_lens), hq, d, max(kv_lens), "cuda", keys_per_split=256)
        ref = A.decode_attention(q, k, v, bt, kl, hq, hkv, d, ws)
        rc, out = _call(fn, q, k, v, bt, kl, hq, hkv, d, ws.keys_per_split, ws.max_splits)
        assert rc == 0, f"call {call}: rc={rc}"
        torch.testing.assert_close(out.float(), ref.float(), atol=2e-2, rtol=2e-2)
        # fp32 oracle on the CPU; the empty-context rows must be exact zeros
        B = len(kv_lens)
        cu = torch.arange(B + 1, dtype=torch.int32)
        oracle = A.paged_attention_ref(q.float().cpu().view(B, hq, d), k.float().cpu(), v.float().cpu(), bt.cpu(),
                                       cu, kl.cpu(), 1.0 / math.sqrt(d), True).view(B, hq * d)
        for b, n in enumerate(kv_lens):
            if n == 0:
                assert torch.all(out[b] == 0), f"call {call}: empty-context row {b} is not zero"
                oracle[b] = 0
        torch.testing.assert_close(out.float().cpu(), oracle, atol=2e-2, rtol=2e-2)


@pytest.mark.gpu
def test_noalloc_decode_rejects_oversized():
    fn = _lib()
    q, k, v, bt, kl = _case([64], 32, 4, 128, 13)
    # 4096 requests x 32 heads x 64 splits x 128 dims is far beyond the static scratch
    rc = fn(q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), bt.data_ptr(), bt.stride(0), kl.data_ptr(),
            4096, 32, 4, 128, 0.1, 256, 64, k.shape[0], q.data_ptr(), q.stride(0),
            torch.cuda.current_stream().cuda_stream)
    assert rc == -1


@pytest.mark.gpu
def test_noalloc_decode_rejects_invalid_arguments():
    fn = _lib()
    hq, hkv, d = 32, 4, 128
    q, k, v, bt, kl = _case([64, 100], hq, hkv, d, 14)
    # (num_heads, num_kv_heads, head_dim, keys_per_split, max_splits, num_pages): each is refused
    # before a launch (a zero KV-head count would otherwise divide by zero on the host)
    for heads, kv_heads, hd, kps, splits, pages in [(hq, 0, d, 256, 4, k.shape[0]), (0, hkv, d, 256, 4, k.shape[0]),
                                                    (hq, 5, d, 256, 4, k.shape[0]), (hq, hkv, d, 0, 4, k.shape[0]),
                                                    (hq, hkv, d, 100, 4, k.shape[0]), (hq, hkv, 96, 256, 4, k.shape[0]),
                                                    (hq, hkv, d, 256, 0, k.shape[0]), (hq, hkv, d, 256, 4, 0)]:
        out = torch.zeros(2, hq * d, dtype=torch.bfloat16, device="cuda")
        rc = fn(q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), bt.data_ptr(), bt.stride(0), kl.data_ptr(),
                2, heads, kv_heads, hd, 0.1, kps, splits, pages, out.data_ptr(), out.stride(0),
                torch.cuda.current_stream().cuda_stream)
        assert rc == -2, (heads, kv_heads, hd, kps, splits, pages, rc)
    torch.cuda.synchronize()


@pytest.mark.gpu
def test_noalloc_decode_clamps_bad_pages():
    """A block-table entry at or past num_pages reads page 0.  The cache is allocated two pages
    longer than the num_pages passed in, so the out-of-range entries still name allocated memory
    and the check cannot turn into a wild read even if the clamp were missing."""
    fn = _lib()
    hq, hkv, d = 32, 4, 128
    q, k, v, bt, kl = _case([200, 64], hq, hkv, d, 15)
    pad = torch.zeros((2,) + tuple(k.shape[1:]), dtype=k.dtype, device=k.device)
    k2 = torch.cat([k, pad + 1])
    v2 = torch.cat([v, pad - 1])
    n = k.shape[0]
    bad = bt.clone()
    bad[0, 1] = n
    bad[1, 0] = n + 1
    rc, out = _call(fn, q, k2, v2, bad, kl, hq, hkv, d, 256, 4, num_pages=n)
    assert rc == 0
    fixed = bad.clone()
    fixed[0, 1] = 0
    fixed[1, 0] = 0
    rc2, ref = _call(fn, q, k2, v2, fixed, kl, hq, hkv, d, 256, 4, num_pages=n)
    assert rc2 == 0
    torch.testing.assert_close(out.float(), ref.float(), atol=0, rtol=0)
