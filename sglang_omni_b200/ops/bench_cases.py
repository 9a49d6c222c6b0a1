"""Small standalone kernel workloads for profiling (one kernel family per case,
three launches, a few GB on the device at most):

    python -m sglang_omni_b200.ops.bench_cases {moe_w13|dense_prefill|decode_attn}

Used to produce the ncu summaries of the hot kernels.
"""
from __future__ import annotations

import sys

import torch

from . import attention as A
from . import gemm as L


def run(case: str) -> None:
    torch.manual_seed(0)
    if case == "moe_w13":
        E, H, I, rows = 128, 2048, 768, 512
        counts = torch.multinomial(torch.ones(E), rows, replacement=True).bincount(minlength=E)
        offs = torch.zeros(E + 1, dtype=torch.int32)
        offs[1:] = counts.cumsum(0)
        offs = offs.cuda()
        x = torch.randn(rows, H, device="cuda").bfloat16()
        w = (torch.randn(E, 2 * I, H, device="cuda") * 0.02).bfloat16()
        h = torch.empty(rows, I, device="cuda", dtype=torch.bfloat16)
        for _ in range(3):
            L.grouped_linear(x, w, offs, gated=True, out=h, expected_rows=rows // E)
    elif case == "dense_prefill":
        x = torch.randn(8192, 2048, device="cuda").bfloat16()
        w = (torch.randn(5120, 2048, device="cuda") * 0.02).bfloat16()
        for _ in range(3):
            L.linear(x, w)
    elif case == "decode_attn":
        B, hq, hkv, d, ctx = 64, 32, 4, 128, 1152
        pages = (ctx + 63) // 64
        k = torch.randn(B * pages + 1, hkv, 64, d, device="cuda").bfloat16()
        v = torch.randn_like(k)
        bt = torch.arange(B * pages, dtype=torch.int32, device="cuda").view(B, pages)
        kl = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
        q = torch.randn(B, hq * d, device="cuda").bfloat16()
        ws = A.DecodeWorkspace(B, hq, d, ctx, "cuda")
        for _ in range(3):
            A.decode_attention(q, k, v, bt, kl, hq, hkv, d, ws)
    else:
        raise SystemExit(f"unknown case {case!r}")
    torch.cuda.synchronize()
    print("ok", case)


if __name__ == "__main__":
    run(sys.argv[1])
