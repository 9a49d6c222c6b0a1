"""Per-kernel device-time breakdown of one thinker serving round (diagnosis).

    python -m sglang_omni_b200.profiler.kernel_breakdown [--requests 64] [--prompt-len 1024]
                                                          [--output-len 256] [--layers 48]

Runs the paged engine on the full Qwen3-Omni thinker architecture (random
weights), two warm-up rounds, one round timed with CUDA events (split into the
prefill phase and the decode phase), then one more round under the CUDA
activity profiler whose kernel records are summed by kernel name.  Kernel
durations under programmatic dependent launch include the time a kernel waited
for its predecessor, so shares of overlapping kernels add up to more than the
round; the CUDA-event times are the ones to quote.
"""
from __future__ import annotations

import argparse
import collections

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--prompt-len", type=int, default=1024)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--top", type=int, default=30)
    args = ap.parse_args()
    from torch.autograd import DeviceType
    from torch.profiler import ProfilerActivity, profile

    from ..engines.ar import AREngine, ARRequest, KVPool
    from ..models.qwen3_omni import loader
    from ..models.qwen3_omni.hf_config import thinker_text_config
    from ..sampling_params import SamplingParams

    R, P, O = args.requests, args.prompt_len, args.output_len
    dev = torch.device("cuda", 0)
    cfg = thinker_text_config(num_layers=args.layers)
    model = loader.get_thinker("random", dev, {"thinker": {"num_layers": args.layers}} if args.layers != 48 else None)
    max_ctx = ((P + O + 63) // 64) * 64
    pool = KVPool(cfg.num_layers, model.cfg.num_kv_heads, cfg.head_dim, R * (max_ctx // 64) + 65, dev)
    eng = AREngine(model, pool, max_batch=R, max_prefill_tokens=8192, max_context=max_ctx, use_graphs=True)
    g = torch.Generator().manual_seed(1234)
    prompts = torch.randint(0, cfg.vocab_size, (R, P), generator=g, dtype=torch.int32).tolist()
    sp = SamplingParams(temperature=0.0, ignore_eos=True)

    def round_(tag, marks=None):
        reqs = [ARRequest(rid=f"{tag}-{i}", prompt_ids=prompts[i], sampling=sp, max_new_tokens=O) for i in range(R)]
        for r in reqs:
            eng.add_request(r)
        while eng.has_work():
            eng.step()
            if marks is not None and not marks and not eng.waiting and not eng.prefilling:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                marks.append(e)

    round_("w0")
    round_("w1")
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    marks: list = []
    s.record()
    round_("t", marks)
    e.record()
    torch.cuda.synchronize()
    print(f"round {s.elapsed_time(e):.1f} ms; prefill phase {s.elapsed_time(marks[0]):.1f} ms; "
          f"decode phase {marks[0].elapsed_time(e):.1f} ms ({marks[0].elapsed_time(e) / O:.2f} ms per step)")
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        round_("p")
        torch.cuda.synchronize()
    agg = collections.defaultdict(lambda: [0, 0.0])
    for ev in prof.events():
        if ev.device_type != DeviceType.CUDA:
            continue
        k = ev.name[:100]
        agg[k][0] += 1
        agg[k][1] += ev.device_time_total
    tot = sum(v[1] for v in agg.values())
    print(f"kernel time under the profiler {tot / 1e3:.1f} ms")
    for k, (n, t) in sorted(agg.items(), key=lambda kv: -kv[1][1])[: args.top]:
        print(f"{t / 1e3:9.2f} ms {100 * t / tot:5.1f}% n={n:7d} avg={t / max(n, 1):8.2f} us  {k}")


if __name__ == "__main__":
    main()
