"""Allocation-free decode attention (C symbol omni_attention_decode_noalloc).

Callers that cannot allocate device memory (a stream capture owned by another
library, host runtimes that pass only inputs and outputs, custom allocators)
use this entry point; its split-KV scratch is a static device array inside the
library.  The test calls the exported C symbol through ctypes and compares its
output with the torch entry point's (which takes a caller-allocated
workspace), on two calls in a row with different inputs, so a stale scratch
from the first call would show up in the second.  This file is collected last
on purpose.
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
                   ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p]
    return fn


def _case(kv_lens, hq, hkv, d, seed):
    g = torch.Generator().manual_seed(seed)
    pages = [(n + 63) // 64 for n in kv_lens]
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


def _call(fn, q, k, v, bt, kl, hq, hkv, d, kps, splits):
    out = torch.full((q.shape[0], hq * d), float("nan"), dtype=torch.bfloat16, device="cuda")
    rc = fn(q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), bt.data_ptr(), bt.stride(0), kl.data_ptr(),
            q.shape[0], hq, hkv, d, 1.0 / math.sqrt(d), kps, splits, out.data_ptr(), out.stride(0),
            torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc, out


@pytest.mark.gpu
def test_noalloc_decode_matches_torch_entry():
    from sglang_omni_b200.ops import attention as A

    fn = _lib()
    hq, hkv, d = 32, 4, 128
    for call, (kv_lens, seed) in enumerate([([1, 700, 64, 1500], 11), ([2000, 3, 129], 12)]):
        q, k, v, bt, kl = _case(kv_lens, hq, hkv, d, seed)
        ws = A.DecodeWorkspace(len(kv_lens), hq, d, max(kv_lens), "cuda", keys_per_split=256)
        ref = A.decode_attention(q, k, v, bt, kl, hq, hkv, d, ws)
        rc, out = _call(fn, q, k, v, bt, kl, hq, hkv, d, ws.keys_per_split, ws.max_splits)
        assert rc == 0, f"call {call}: rc={rc}"
        torch.testing.assert_close(out.float(), ref.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.gpu
def test_noalloc_decode_rejects_oversized():
    fn = _lib()
    q, k, v, bt, kl = _case([64], 32, 4, 128, 13)
    # 4096 requests x 32 heads x 64 splits x 128 dims is far beyond the static scratch
    rc = fn(q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), bt.data_ptr(), bt.stride(0), kl.data_ptr(),
            4096, 32, 4, 128, 0.1, 256, 64, q.data_ptr(), q.stride(0), torch.cuda.current_stream().cuda_stream)
    assert rc == -1
