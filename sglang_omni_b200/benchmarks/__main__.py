"""Command line of the serving benchmarks (see the package docstring for examples).

Each run waits for ``GET /health``, sends ``--warmup`` requests one at a time, then the samples
at every concurrency of ``--concurrency`` (comma-separated), prints one summary row per
concurrency and writes ``<output-dir>/<task>.json`` (summaries and per-request outcomes).
``--baseline FILE`` (JSON {metric: value} or {concurrency: {metric: value}}) exits non-zero when
a metric regresses past the 0.75x / 1.25x gate."""
from __future__ import annotations

import argparse
import asyncio
import json
import math
import os
import sys
import time

from .datasets import load_meta_lst, synthetic_samples
from .results import regression_failures, summarize
from .runner import run_requests


def wait_healthy(base_url: str, timeout_s: float) -> None:
    import httpx

    t0 = time.time()
    while True:
        try:
            if httpx.get(f"{base_url}/health", timeout=2.0).status_code == 200:
                return
        except httpx.HTTPError:
            pass
        if time.time() - t0 > timeout_s:
            raise SystemExit(f"{base_url} not healthy after {timeout_s:.0f} s")
        time.sleep(1.0)


def _samples(a):
    if a.testset:
        return load_meta_lst(a.testset, a.max_samples)
    return synthetic_samples(a.max_samples or 16, seed=a.seed)


def _sender(a, save_dir):
    from . import senders

    params = {"max_new_tokens": a.max_new_tokens, "temperature": a.temperature, "top_p": a.top_p,
              "top_k": a.top_k, "repetition_penalty": a.repetition_penalty}
    if a.task == "omni-speed":
        async def send(session, sample, i):
            return await senders.omni_chat(session, a.base_url, sample, f"{a.task}-{i}", model=a.model,
                                           stream=a.stream, lang=a.lang, max_tokens=a.max_tokens,
                                           temperature=a.temperature if a.temperature is not None else 0.7,
                                           use_reference=not a.no_ref_audio, save_dir=save_dir)
    else:
        async def send(session, sample, i):
            return await senders.speech(session, a.base_url, sample, f"{a.task}-{i}", model=a.model,
                                        stream=a.stream, params=params, use_reference=not a.no_ref_audio,
                                        save_dir=save_dir)
    return send


async def _run_level(a, samples, conc: int, save_dir):
    import aiohttp

    send = _sender(a, save_dir)
    async with aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=a.request_timeout)) as session:
        outcomes, wall = await run_requests(samples, lambda s, i: send(session, s, i), concurrency=conc,
                                            rate=a.request_rate, warmup=a.warmup)
    return outcomes, wall


def _row(conc: int, s: dict) -> str:
    keys = ("completed_requests", "failed_requests", "latency_mean_s", "latency_p95_s", "ttfa_median_s",
            "rtf_mean", "throughput_qps", "tok_per_s_agg", "audio_s_per_s")
    return f"c={conc:<4d} " + "  ".join(f"{k}={s[k]}" for k in keys if k in s)


def _wer(a, results: dict) -> None:
    from ..client.audio import decode_wav
    from .wer import load_asr, score, wer_summary

    asr = load_asr(a.asr, a.asr_device)
    for level in results["levels"]:
        aligns = []
        for o in level["outcomes"]:
            if not o["ok"] or not o["wav_path"]:
                aligns.append(None)
                continue
            with open(o["wav_path"], "rb") as f:
                wave, rate = decode_wav(f.read())
            hyp = asr(wave, rate, a.lang)
            al = score(o["text"], hyp, a.lang)
            o["asr_text"], o["wer"] = hyp, al.rate
            aligns.append(al)
        level["wer"] = wer_summary(aligns, a.lang)
        print(f"c={level['concurrency']:<4d} " + "  ".join(f"{k}={v}" for k, v in level["wer"].items()))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m sglang_omni_b200.benchmarks")
    ap.add_argument("task", choices=["tts-speed", "omni-speed", "tts-wer"])
    ap.add_argument("--base-url", default=None, help="e.g. http://127.0.0.1:8000 (overrides --host / --port)")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--model", default="default")
    ap.add_argument("--testset", default=None, help="seed-tts-eval meta.lst (default: synthetic sentences)")
    ap.add_argument("--max-samples", type=int, default=None)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-ref-audio", action="store_true", help="plain TTS: ignore the testset's reference clips")
    ap.add_argument("--concurrency", default="1", help="comma-separated levels, e.g. 1,2,4,8,16")
    ap.add_argument("--request-rate", type=float, default=math.inf, help="Poisson arrivals per second (inf: all)")
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--stream", action="store_true", help="streamed responses (time to first audio)")
    ap.add_argument("--max-new-tokens", type=int, default=None)
    ap.add_argument("--max-tokens", type=int, default=256, help="omni-speed: thinker tokens")
    ap.add_argument("--temperature", type=float, default=None)
    ap.add_argument("--top-p", type=float, default=None)
    ap.add_argument("--top-k", type=int, default=None)
    ap.add_argument("--repetition-penalty", type=float, default=None)
    ap.add_argument("--lang", default="en", choices=["en", "zh"])
    ap.add_argument("--asr", default=None, help="tts-wer: whisper:<dir> or module:function")
    ap.add_argument("--asr-device", default="cpu")
    ap.add_argument("--save-audio", action="store_true")
    ap.add_argument("--output-dir", default="results/benchmarks")
    ap.add_argument("--baseline", default=None)
    ap.add_argument("--request-timeout", type=float, default=600.0)
    ap.add_argument("--wait-timeout", type=float, default=1200.0)
    a = ap.parse_args(argv)
    a.base_url = (a.base_url or f"http://{a.host}:{a.port}").rstrip("/")
    if a.task == "tts-wer" and not a.asr:
        ap.error("tts-wer needs --asr")
    wait_healthy(a.base_url, a.wait_timeout)
    samples = _samples(a)
    os.makedirs(a.output_dir, exist_ok=True)
    save = a.save_audio or a.task == "tts-wer"
    results = {"task": a.task, "base_url": a.base_url, "model": a.model, "stream": a.stream,
               "samples": len(samples), "levels": []}
    for conc in [int(c) for c in a.concurrency.split(",") if c.strip()]:
        save_dir = os.path.join(a.output_dir, f"{a.task}-c{conc}-audio") if save else None
        outcomes, wall = asyncio.run(_run_level(a, samples, conc, save_dir))
        summ = summarize(outcomes, wall)
        print(_row(conc, summ), flush=True)
        results["levels"].append({"concurrency": conc, "wall_s": wall, "summary": summ,
                                  "outcomes": [o.to_dict() for o in outcomes]})
    if a.task == "tts-wer":
        _wer(a, results)
    with open(os.path.join(a.output_dir, f"{a.task}.json"), "w") as f:
        json.dump(results, f, indent=1)
    if a.baseline:
        with open(a.baseline) as f:
            base = json.load(f)
        bad = []
        for level in results["levels"]:
            ref = base.get(str(level["concurrency"]), base)
            bad += [f"c={level['concurrency']} {m}" for m in regression_failures(level["summary"], ref)]
        if bad:
            print("regressions:\n  " + "\n  ".join(bad), file=sys.stderr)
            return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
