"""Timing of the fused compute + collective paths against their NCCL baselines and rooflines.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m sglang_omni_b200.parallel.bench_fused

One process per GPU.  Every time is CUDA-event device time on the launching stream
after warm-up, averaged over ``--iters`` iterations, the max over ranks.

* TP reduce point (the thinker's o_proj at TP=N): the o_proj GEMM whose epilogue
  stores every output row into its owner rank's partial slot (NVLink stores from
  the GEMM) + the reduce / residual / RMSNorm / all-gather kernel, against the
  NCCL baseline (plain GEMM, ``all_reduce``, RMSNorm).  Roofline: the slower of
  the GEMM FLOPs at the measured sustained bf16 rate and the bytes each GPU must
  send (its (N-1)/N partial rows + (N-1) copies of its normalised owned rows) at
  the measured 770 GB/s per direction.
* EP MoE layer (128 experts, top-8, hidden 2048, expert width 768 at EP=N): router
  and top-k, dispatch straight into the owners' expert segments, the grouped GEMMs
  (w13 waits for the dispatch flags itself, the w2 epilogue stores the rows into
  the source ranks' slots), the top-k weighted sum waiting for the owners' flags;
  against the NCCL all-to-all dispatcher (count all-to-all + host copy of the split
  sizes, ``all_to_all_single`` of the rows both ways, the same grouped GEMMs).
  Roofline: the slowest of this rank's expert weights at the measured HBM copy
  rate, the expert GEMM FLOPs at the sustained bf16 rate and the dispatched +
  combined rows at 770 GB/s.
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

HBM_GBS = 6546.9          # measured copy bandwidth (B200)
BF16_TFLOPS = 1395.6      # measured sustained cuBLAS bf16
NVLINK_GBS = 770.0        # measured peer copy per direction


def _time(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters * 1e3], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0])


def tp_reduce_point(T: int, iters: int, rank: int, world: int) -> dict:
    from ..ops import gemm, norm
    from .tp import TPGroup

    H, K = 2048, 4096 // world            # o_proj columns of this rank's heads
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(T, K, device=dev, generator=g).bfloat16()
    w = (torch.randn(H, K, device=dev, generator=g) * 0.02).bfloat16()
    nw = torch.ones(H, device=dev).bfloat16()
    res = torch.randn(T, H, device=dev, generator=g).bfloat16()
    tp = TPGroup(H, T, dev)
    part = torch.empty(T, H, device=dev, dtype=torch.bfloat16)

    def fused():
        # the producer GEMM waits (in its TMA thread) for every owner's previous all-gather
        # phase before overwriting their partial slots, as the decoder's GEMMs do
        with gemm.static_weights():
            gemm.linear(x, w, out=tp.part_local[:T], scatter=tp.scatter(T), wait=tp.wait)
        tp.reduce_norm(res, nw, 1e-6, T)

    def nccl():
        gemm.linear(x, w, out=part)
        dist.all_reduce(part)
        norm.rms_norm(part, nw, 1e-6, residual=res)

    t_f = _time(fused, iters)
    t_n = _time(nccl, iters)
    tp.close()
    flops = 2.0 * T * K * H
    send = T * H * 2 * (world - 1) / world * 2          # partial rows out + normalised rows to every peer
    roof = max(flops / (BF16_TFLOPS * 1e6), send / (NVLINK_GBS * 1e3))
    return {"path": "TP o_proj GEMM -> reduce-scatter + residual + RMSNorm + all-gather", "tokens": T,
            "fused_us": round(t_f, 2), "nccl_us": round(t_n, 2), "roofline_us": round(roof, 2),
            "fused_frac_of_roofline": round(roof / t_f, 3), "speedup_vs_nccl": round(t_n / t_f, 3)}


class _NcclEP:
    """NCCL baseline of one EP MoE layer (the all-to-all token dispatcher of Megatron-style EP):
    route, permute the rows by expert locally, exchange the per-expert counts with an
    all-to-all, copy them to the host (the variable split sizes of the next all-to-all), send
    the rows with ``all_to_all_single``, reorder them expert-major, run the same grouped
    GEMMs, undo the reorder, send the outputs back and do the top-k weighted sum."""

    def __init__(self, E, topk, H, I, T, world, rank, dev):
        from ..ops.moe import MoEWorkspace

        self.E, self.topk, self.H, self.I, self.world, self.rank = E, topk, H, I, world, rank
        self.El = E // world
        self.ws = MoEWorkspace(T, E, topk, H, I, dev)
        self.dev = dev

    def forward(self, x, wr, w13, w2, out):
        from ..ops import gemm
        from ..ops._ext import ext
        from ..ops.moe import route

        T, k, El, W = x.shape[0], self.topk, self.El, self.world
        ws = self.ws
        logits = gemm.linear(x, wr, out_dtype=torch.float32)
        route(logits, k, ws=ws, x=x)                        # ids, weights, offsets, inv_perm, x_perm (expert-major)
        cnt = (ws.offsets[1:] - ws.offsets[:-1]).view(W, El)  # rows of this rank for each (destination, expert)
        rcnt = torch.empty_like(cnt)
        dist.all_to_all_single(rcnt, cnt)                    # rows each source sends to my experts
        c_send, c_recv = cnt.cpu(), rcnt.cpu()               # host sync: the split sizes
        send = c_send.sum(1).tolist()
        recv = c_recv.sum(1).tolist()
        rows_in = sum(recv)
        xr = torch.empty(rows_in, self.H, dtype=x.dtype, device=self.dev)
        dist.all_to_all_single(xr, ws.x_perm[: T * k], recv, send)
        # source-major [s][e] blocks -> expert-major [e][s]
        starts = torch.cumsum(torch.cat([torch.zeros(1, dtype=torch.long), c_recv.flatten()]), 0)
        idx = torch.cat([torch.arange(int(starts[s * El + e]), int(starts[s * El + e + 1]))
                         for e in range(El) for s in range(W)]) if rows_in else torch.zeros(0, dtype=torch.long)
        idx = idx.to(self.dev, non_blocking=True)
        offs = torch.cat([torch.zeros(1, dtype=torch.long), torch.cumsum(c_recv.sum(0), 0)]).to(torch.int32)
        offs = offs.to(self.dev, non_blocking=True)
        xe = xr.index_select(0, idx)
        h = gemm.grouped_linear(xe, w13, offs, gated=True, expected_rows=max(1, rows_in // El))
        ye = gemm.grouped_linear(h, w2, offs, expected_rows=max(1, rows_in // El))
        yr = torch.empty_like(xr)
        yr.index_copy_(0, idx, ye)
        yb = torch.empty(T * k, self.H, dtype=x.dtype, device=self.dev)
        dist.all_to_all_single(yb, yr, send, recv)
        ext().moe_combine(yb, ws.inv_perm[:T], ws.topk_w[:T], out, None, None)
        return out


def ep_moe_layer(T: int, iters: int, rank: int, world: int) -> dict:
    from .ep_moe import EPMoE

    E, topk, H, I = 128, 8, 2048, 768
    El = E // world
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(T, H, device=dev, generator=g).bfloat16()
    wr = (torch.randn(E, H, device=dev, generator=torch.Generator(device=dev).manual_seed(0)) * 0.02).bfloat16()
    w13 = (torch.randn(El, 2 * I, H, device=dev, generator=g) * 0.02).bfloat16()
    w2 = (torch.randn(El, H, I, device=dev, generator=g) * 0.02).bfloat16()
    ep = EPMoE(E, topk, H, I, max_tokens=T, device=dev)
    out = torch.empty_like(x)
    t_f = _time(lambda: ep.forward(x, wr, w13, w2, out=out), iters)
    ref = _NcclEP(E, topk, H, I, T, world, rank, dev)
    out_n = torch.empty_like(x)
    t_n = _time(lambda: ref.forward(x, wr, w13, w2, out_n), iters)
    ep.forward(x, wr, w13, w2, out=out)
    torch.cuda.synchronize()
    err = float((out.float() - out_n.float()).norm() / out_n.float().norm().clamp_min(1e-6))
    # per-kernel device time inside the layer: an event after every launch
    names: list = []
    stamps: list = []

    class _Marks(list):
        def append(self, name):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            names.append(name)
            stamps.append(ev)

    parts: dict = {}
    for _ in range(iters):
        names.clear()
        stamps.clear()
        # keep the GPU busy while the host enqueues the layer, so the events time the device only
        torch.cuda._sleep(2_000_000)
        e0 = torch.cuda.Event(enable_timing=True)
        e0.record()
        ep._marks = _Marks()
        ep.forward(x, wr, w13, w2, out=out)
        ep._marks = None
        torch.cuda.synchronize()
        prev = e0
        for nm, ev in zip(names, stamps):
            parts[nm] = parts.get(nm, 0.0) + prev.elapsed_time(ev) * 1e3 / iters
            prev = ev
    pt = torch.tensor([parts[n] for n in names], dtype=torch.float64, device=dev)
    dist.all_reduce(pt, op=dist.ReduceOp.MAX)
    breakdown = {n: round(float(v), 2) for n, v in zip(names, pt)}
    ep.close()
    wbytes = El * 3 * H * I * 2
    flops = T * topk * 2.0 * 3 * H * I                    # rows landing on this rank (T * topk on average)
    rows = T * topk * (world - 1) / world                 # (token, k) rows that leave this rank
    link = rows * H * 2 * 2                                # dispatched and combined back
    roof = max(wbytes / (HBM_GBS * 1e3), flops / (BF16_TFLOPS * 1e6), link / (NVLINK_GBS * 1e3))
    return {"path": "EP MoE layer: router + top-k, dispatch into the owners' expert segments (system-atomic "
                    "reservations), w13 GEMM waiting on the dispatch flags, w2 GEMM storing rows into the "
                    "source ranks' slots, combine waiting on the owners' flags", "tokens_per_rank": T,
            "fused_us": round(t_f, 2), "nccl_us": round(t_n, 2), "roofline_us": round(roof, 2),
            "fused_frac_of_roofline": round(roof / t_f, 3), "speedup_vs_nccl": round(t_n / t_f, 3),
            "rel_diff_vs_nccl": round(err, 4), "breakdown_us_max_over_ranks": breakdown}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--paths", default="tp,ep", help="comma list of tp, ep")
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    from datetime import timedelta

    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=300))
    rank, world = dist.get_rank(), dist.get_world_size()
    from ..ops import _ext

    _ext.ext()
    rows = []
    paths = args.paths.split(",")
    if "tp" in paths:
        for T in (64, 8192):
            rows.append(tp_reduce_point(T, args.iters, rank, world))
    if "ep" in paths:
        for T in (64, 2048):
            rows.append(ep_moe_layer(T, args.iters, rank, world))
    _ext.check_status(torch.device("cuda", local))
    if rank == 0:
        for r in rows:
            print(json.dumps({"world": world, **r}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
