"""Small standalone kernel workloads for profiling (one kernel family per case,
three launches, a few GB on the device at most):

    python -m sglang_omni_b200.ops.bench_cases {moe_w13|dense_prefill|decode_attn|decode_dense|
                                                prefill_attn|rmsnorm|rope_store|moe_route|sample|time|
                                                code2wav}

Used to produce the ncu summaries of the hot kernels.
"""
from __future__ import annotations

import os
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
    elif case == "decode_dense":
        # thinker decode projections at batch 64: QKV, o_proj, router (fp32 logits); split-K path
        x = torch.randn(64, 2048, device="cuda").bfloat16()
        xo = torch.randn(64, 4096, device="cuda").bfloat16()
        wq = (torch.randn(5120, 2048, device="cuda") * 0.02).bfloat16()
        wo = (torch.randn(2048, 4096, device="cuda") * 0.02).bfloat16()
        wr = (torch.randn(128, 2048, device="cuda") * 0.02).bfloat16()
        for _ in range(3):
            L.linear(x, wq)
            L.linear(xo, wo)
            L.linear(x, wr, out_dtype=torch.float32)
    elif case == "prefill_attn":
        # one 8192-token prefill chunk: 8 requests x 1024 prompt tokens, 32 q / 4 kv heads x 128, causal
        from . import prefill_tiles
        R, P, hq, hkv, d = 8, 1024, 32, 4, 128
        pages = P // 64
        k = torch.randn(R * pages + 1, hkv, 64, d, device="cuda").bfloat16()
        v = torch.randn_like(k)
        bt = torch.arange(1, R * pages + 1, dtype=torch.int32, device="cuda").view(R, pages)
        kl = torch.full((R,), P, dtype=torch.int32, device="cuda")
        cu = torch.arange(0, R * P + 1, P, dtype=torch.int32, device="cuda")
        rows = int(os.environ.get("OMNI_BENCH_TILE_ROWS", "256"))   # 256 / 128: tcgen05 kernels, 64: mma.sync
        tr, t0 = prefill_tiles([P] * R, hq // hkv, rows)
        tr = torch.tensor(tr, dtype=torch.int32, device="cuda")
        t0 = torch.tensor(t0, dtype=torch.int32, device="cuda")
        q = torch.randn(R * P, hq * d, device="cuda").bfloat16()
        for _ in range(3):
            A.prefill_attention(q, k, v, bt, cu, kl, tr, t0, hq, hkv, d, tile_rows=rows)
    elif case == "rmsnorm":
        # fused residual add + RMSNorm over 65536 x 2048 bf16 (268 MB per tensor, > L2)
        from .norm import rms_norm
        x = torch.randn(65536, 2048, device="cuda").bfloat16()
        r = torch.randn_like(x)
        w = torch.randn(2048, device="cuda").bfloat16()
        out = torch.empty_like(x)
        for _ in range(3):
            rms_norm(x, w, 1e-6, residual=r, out=out)
    elif case == "rope_store":
        # QK-RMSNorm + interleaved M-RoPE + paged KV store, 65536 tokens x (32 + 2 x 4) heads x 128
        from .rope import qkv_rope_store, rope_tables
        T, hq, hkv, d = 65536, 32, 4, 128
        qkv = torch.randn(T, (hq + 2 * hkv) * d, device="cuda").bfloat16()
        cos, sin = rope_tables(d, 1e6, 8192, "cuda")
        pos = torch.randint(0, 8192, (3, T), dtype=torch.int32, device="cuda")
        kc = torch.zeros(T // 64 + 1, hkv, 64, d, device="cuda").bfloat16()
        vc = torch.zeros_like(kc)
        slots = torch.arange(64, T + 64, dtype=torch.int32, device="cuda")
        qn = torch.ones(d, device="cuda").bfloat16()
        for _ in range(3):
            qkv_rope_store(qkv, hq, hkv, d, pos, cos, sin, q_norm=qn, k_norm=qn, mrope_section=[24, 20, 20],
                           slot_mapping=slots, k_cache=kc, v_cache=vc)
    elif case == "rope_decode":
        # the decode-step shape: 64 tokens x (32 + 2 x 4) heads x 128, M-RoPE, paged KV store
        from .rope import qkv_rope_store, rope_tables
        T, hq, hkv, d = 64, 32, 4, 128
        qkv = torch.randn(T, (hq + 2 * hkv) * d, device="cuda").bfloat16()
        cos, sin = rope_tables(d, 1e6, 8192, "cuda")
        pos = torch.randint(0, 8192, (3, T), dtype=torch.int32, device="cuda")
        kc = torch.zeros(1025, hkv, 64, d, device="cuda").bfloat16()
        vc = torch.zeros_like(kc)
        slots = torch.randint(64, 1025 * 64, (T,), dtype=torch.int32, device="cuda")
        qn = torch.ones(d, device="cuda").bfloat16()
        for _ in range(3):
            qkv_rope_store(qkv, hq, hkv, d, pos, cos, sin, q_norm=qn, k_norm=qn, mrope_section=[24, 20, 20],
                           slot_mapping=slots, k_cache=kc, v_cache=vc)
    elif case == "moe_route":
        # softmax top-8 of 128 experts + expert histogram / offsets + permuted gather of 8192 x 2048 rows
        from .moe import MoEWorkspace, route
        T, E, H = 8192, 128, 2048
        ws = MoEWorkspace(T, E, 8, H, 768, "cuda")
        logits = torch.randn(T, E, device="cuda")
        x = torch.randn(T, H, device="cuda").bfloat16()
        for _ in range(3):
            route(logits, 8, ws=ws, x=x)
    elif case == "sample":
        # top-k 50 / top-p 0.9 / temperature 0.8 sampling of 64 x 151936 fp32 logits
        from .sampling import SamplingTensors, sample
        B, V = 64, 151936
        logits = torch.randn(B, V, device="cuda")
        st = SamplingTensors(torch.full((B,), 0.8, device="cuda"), torch.full((B,), 50, dtype=torch.int32, device="cuda"),
                             torch.full((B,), 0.9, device="cuda"), torch.zeros(B, device="cuda"))
        for _ in range(3):
            sample(logits.clone(), st)
    elif case == "time":
        _time_cases()
        return
    elif case == "code2wav":
        _code2wav_chunk()
        return
    else:
        raise SystemExit(f"unknown case {case!r}")
    torch.cuda.synchronize()
    print("ok", case)


def _time_cases() -> None:
    """CUDA-event times of the decode-step kernels in isolation (L2 flushed between iterations)."""
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")

    def t(fn, n=20):
        for _ in range(3):
            fn()
        tot = 0.0
        for _ in range(n):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            # keep the GPU busy while the host enqueues fn, so the events time the device only
            torch.cuda._sleep(200_000)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            tot += a.elapsed_time(b)
        return tot / n * 1e3

    x = torch.randn(64, 2048, device="cuda").bfloat16()
    xo = torch.randn(64, 4096, device="cuda").bfloat16()
    wq = (torch.randn(5120, 2048, device="cuda") * 0.02).bfloat16()
    wo = (torch.randn(2048, 4096, device="cuda") * 0.02).bfloat16()
    wr = (torch.randn(128, 2048, device="cuda") * 0.02).bfloat16()
    wl = (torch.randn(151936, 2048, device="cuda") * 0.02).bfloat16()
    res = {
        "qkv 5120x2048 T64": (t(lambda: L.linear(x, wq)), wq.numel() * 2),
        "o_proj 2048x4096 T64": (t(lambda: L.linear(xo, wo)), wo.numel() * 2),
        "router 128x2048 T64 fp32": (t(lambda: L.linear(x, wr, out_dtype=torch.float32)), wr.numel() * 2),
        "lm_head 151936x2048 T64 fp32": (t(lambda: L.linear(x, wl, out_dtype=torch.float32)), wl.numel() * 2),
    }
    import torch.nn.functional as F
    flops = {}
    xp = torch.randn(8192, 2048, device="cuda").bfloat16()
    xo = torch.randn(8192, 4096, device="cuda").bfloat16()
    for name, (xx, ww) in {"qkv prefill 8192x2048 -> 5120": (xp, wq), "o_proj prefill 8192x4096 -> 2048": (xo, wo)}.items():
        f = 2.0 * xx.shape[0] * xx.shape[1] * ww.shape[0]
        flops[name] = (t(lambda: L.linear(xx, ww)), f)
        flops[name + " (cuBLAS)"] = (t(lambda: F.linear(xx, ww)), f)
    # encoder GEMMs: vision tower (64 images x 784 patches, d 1152, MLP 4304, QKV padded to 80 / head)
    # and audio tower (32 x 10 s -> 4160 tokens, d 1280, MLP 5120)
    enc = {
        "vision qkv 50176x1152 -> 3840": (50176, 1152, 3840),
        "vision fc1 50176x1152 -> 4304": (50176, 1152, 4304),
        "vision fc2 50176x4304 -> 1152": (50176, 4304, 1152),
        "audio qkv 4160x1280 -> 3840": (4160, 1280, 3840),
        "audio fc1 4160x1280 -> 5120": (4160, 1280, 5120),
    }
    for name, (M, K, N) in enc.items():
        xx = torch.randn(M, K, device="cuda").bfloat16()
        ww = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
        f = 2.0 * M * K * N
        flops[name] = (t(lambda: L.linear(xx, ww), n=10), f)
        flops[name + " (cuBLAS)"] = (t(lambda: F.linear(xx, ww), n=10), f)
        del xx, ww
    # paged causal prefill attention, 8 x 1024 tokens, 32 q / 4 kv heads x 128 (half the QK^T / PV work is masked)
    from . import prefill_tiles
    R, P, hq, hkv, d = 8, 1024, 32, 4, 128
    pages = P // 64
    k = torch.randn(R * pages + 1, hkv, 64, d, device="cuda").bfloat16()
    v = torch.randn_like(k)
    bt = torch.arange(1, R * pages + 1, dtype=torch.int32, device="cuda").view(R, pages)
    kl = torch.full((R,), P, dtype=torch.int32, device="cuda")
    cu = torch.arange(0, R * P + 1, P, dtype=torch.int32, device="cuda")
    q = torch.randn(R * P, hq * d, device="cuda").bfloat16()
    f_attn = 4.0 * R * (P * (P + 1) / 2) * hq * d   # causal: QK^T + PV over the visible keys
    for rows, tag in ((64, "mma.sync"), (128, "tcgen05"), (256, "tcgen05 2-tile")):
        tr, t0 = prefill_tiles([P] * R, hq // hkv, rows)
        tr = torch.tensor(tr, dtype=torch.int32, device="cuda")
        t0 = torch.tensor(t0, dtype=torch.int32, device="cuda")
        flops[f"prefill attn 8x1024 causal 32/4x128 ({tag})"] = (
            t(lambda: A.prefill_attention(q, k, v, bt, cu, kl, tr, t0, hq, hkv, d, tile_rows=rows)), f_attn)
    for name, (us, f) in flops.items():
        print(f"{name:44s} {us:8.2f} us  {f / us / 1e6:7.1f} TFLOP/s")
    B, hq, hkv, d, ctx = 64, 32, 4, 128, 1152
    pages = (ctx + 63) // 64
    k = torch.randn(B * pages + 1, hkv, 64, d, device="cuda").bfloat16()
    v = torch.randn_like(k)
    bt = torch.arange(B * pages, dtype=torch.int32, device="cuda").view(B, pages)
    kl = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    q = torch.randn(B, hq * d, device="cuda").bfloat16()
    # 64 x 4 (request, KV head) pairs take one split each; 16 requests (64 pairs) split the keys
    for nb in (B, 16):
        ws = A.DecodeWorkspace(nb, hq, d, ctx, "cuda")
        res[f"decode_attn B{nb} ctx1152"] = (t(lambda: A.decode_attention(q[:nb], k, v, bt[:nb], kl[:nb], hq, hkv, d,
                                                                          ws)), 2 * nb * ctx * hkv * d * 2)
    # split sizes of the GPU-filling batch (the rule's FILL_SPLIT_KEYS), B=64 ctx 1152
    fill = A.FILL_SPLIT_KEYS
    for kps in (256, 384, 576):
        A.FILL_SPLIT_KEYS = kps
        ws = A.DecodeWorkspace(B, hq, d, ctx, "cuda", keys_per_split=kps)
        res[f"decode_attn B64 ctx1152 split {kps}"] = (
            t(lambda: A.decode_attention(q, k, v, bt, kl, hq, hkv, d, ws)), 2 * B * ctx * hkv * d * 2)
    A.FILL_SPLIT_KEYS = fill
    # skewed batch: 63 requests at 1152 keys and one at 8192 (its pages follow the others')
    long_pages = 8192 // 64
    ks = torch.randn(B * pages + long_pages + 1, hkv, 64, d, device="cuda").bfloat16()
    vs = torch.randn_like(ks)
    bts = torch.zeros(B, long_pages, dtype=torch.int32, device="cuda")
    bts[:, :pages] = bt
    bts[B - 1] = torch.arange(B * pages, B * pages + long_pages, dtype=torch.int32, device="cuda")
    kls = kl.clone()
    kls[B - 1] = 8192
    ws = A.DecodeWorkspace(B, hq, d, 8192, "cuda")
    res["decode_attn B64 ctx1152 + one 8192"] = (t(lambda: A.decode_attention(q, ks, vs, bts, kls, hq, hkv, d, ws)),
                                                 2 * (63 * ctx + 8192) * hkv * d * 2)
    # memory-bound prefill kernels (inputs larger than L2)
    from .norm import rms_norm
    from .rope import qkv_rope_store, rope_tables

    xn = torch.randn(65536, 2048, device="cuda").bfloat16()
    rn = torch.randn_like(xn)
    wn = torch.randn(2048, device="cuda").bfloat16()
    on = torch.empty_like(xn)
    res["add + RMSNorm 65536x2048"] = (t(lambda: rms_norm(xn, wn, 1e-6, residual=rn, out=on), n=10),
                                       4 * xn.numel() * 2)   # read x, residual; write residual, out
    del xn, rn, on
    T, hq, hkv, d = 65536, 32, 4, 128
    qkv = torch.randn(T, (hq + 2 * hkv) * d, device="cuda").bfloat16()
    cos, sin = rope_tables(d, 1e6, 8192, "cuda")
    pos = torch.randint(0, 8192, (3, T), dtype=torch.int32, device="cuda")
    kc = torch.zeros(T // 64 + 1, hkv, 64, d, device="cuda").bfloat16()
    vc = torch.zeros_like(kc)
    slots = torch.arange(64, T + 64, dtype=torch.int32, device="cuda")
    qn = torch.ones(d, device="cuda").bfloat16()
    res["QK-norm + M-RoPE + KV store 65536 tok"] = (
        t(lambda: qkv_rope_store(qkv, hq, hkv, d, pos, cos, sin, q_norm=qn, k_norm=qn, mrope_section=[24, 20, 20],
                                 slot_mapping=slots, k_cache=kc, v_cache=vc), n=10),
        qkv.numel() * 2 + T * (hq + 2 * hkv) * d * 2)   # read q, k, v rows; write q in place, k / v pages
    for name, (us, nbytes) in res.items():
        print(f"{name:36s} {us:8.2f} us  {nbytes / us / 1e3:7.1f} GB/s")



def _code2wav_chunk(streams: int = 32, chunk: int = 10, context: int = 25) -> None:
    """Released-size Code2Wav (random bf16 weights), one steady streaming chunk of every stream:
    the windowed decode (context + chunk frames per stream, one graph) against the stateful one
    (the chunk's frames only, one graph).  CUDA events, L2 flushed, the GPU kept busy while the
    host enqueues."""
    from ..models.qwen3_omni.code2wav import Code2Wav, Code2WavConfig, Code2WavGraphs
    from ..models.qwen3_omni.code2wav_stateful import StatefulGraphs, Code2WavStreamState

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    m = Code2Wav(Code2WavConfig(), device="cuda").random_init_(seed=0)
    Q = m.cfg.num_quantizers
    codes = torch.randint(0, m.cfg.codebook_size, (streams, Q, context + chunk), device="cuda")
    win = Code2WavGraphs(m, streams)
    win.capture(streams, context + chunk)
    state = Code2WavStreamState(m, streams, 4096, chunk)
    sg = StatefulGraphs(state, streams)
    sg.capture(streams, chunk, False)
    slots = torch.arange(streams, device="cuda")
    with torch.no_grad():   # three chunks of history per stream
        state.step(codes[:, :, :chunk], slots, True)
        for _ in range(2):
            state.step(codes[:, :, :chunk], slots, False)

    def t(fn, n=20):
        for _ in range(3):
            fn()
        tot = 0.0
        for _ in range(n):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda._sleep(200_000)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            tot += a.elapsed_time(b)
        return tot / n * 1e3

    with torch.no_grad():
        tw = t(lambda: win(codes))
        ts = t(lambda: sg(codes[:, :, :chunk], slots, False))
    print(f"code2wav chunk, {streams} streams: windowed ({context}+{chunk} frames) {tw:9.1f} us   "
          f"stateful ({chunk} frames) {ts:9.1f} us   ratio {tw / ts:5.2f}   state {state.state_bytes() / 2**20:.0f} MiB")


if __name__ == "__main__":
    run(sys.argv[1])
