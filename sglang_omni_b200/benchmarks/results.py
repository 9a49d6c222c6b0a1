"""Per-request outcomes, their summary and the regression gate.

Summary keys follow the reference's reported metrics (benchmarks/metrics/performance.py:11-73):
``latency_{mean,median,p95,p99}_s``, ``rtf_{mean,median}``, ``throughput_qps`` (successes per wall
second), ``tok_per_s_agg`` (sum of completion tokens / sum of engine seconds).  Streamed requests
add ``ttfa_{mean,median,p95}_s`` (time to the first audio chunk) and, for chat, ``ttft_*``.
The gate mirrors the reference's CI rule (tests/utils.py:183-201): throughput-like metrics may
fall to 0.75x of a baseline, latency-like ones may rise to 1.25x."""
from __future__ import annotations

from dataclasses import asdict, dataclass, field

import numpy as np


@dataclass
class RequestOutcome:
    request_id: str
    ok: bool = False
    error: str = ""
    latency_s: float = 0.0           # request sent -> response complete
    ttfa_s: float | None = None      # first audio bytes (streamed requests)
    ttft_s: float | None = None      # first text delta (streamed chat)
    audio_s: float = 0.0             # seconds of audio received
    prompt_tokens: int = 0
    completion_tokens: int = 0
    engine_time_s: float = 0.0       # server-side time of the generating stage
    text: str = ""                   # text output (chat) or the synthesised text (speech)
    wav_path: str = ""
    extra: dict = field(default_factory=dict)

    @property
    def rtf(self) -> float | None:
        return self.latency_s / self.audio_s if self.ok and self.audio_s > 0 else None

    @property
    def tok_per_s(self) -> float | None:
        if self.completion_tokens > 0 and self.engine_time_s > 0:
            return self.completion_tokens / self.engine_time_s
        return None

    def to_dict(self) -> dict:
        d = asdict(self)
        d["rtf"], d["tok_per_s"] = self.rtf, self.tok_per_s
        return d


def _stats(prefix: str, xs: list[float], quantiles=(50, 95, 99), digits: int = 4) -> dict:
    if not xs:
        return {}
    a = np.asarray(xs, dtype=np.float64)
    out = {f"{prefix}_mean": round(float(a.mean()), digits)}
    names = {50: "median", 95: "p95", 99: "p99"}
    for q in quantiles:
        out[f"{prefix}_{names[q]}"] = round(float(np.percentile(a, q)), digits)
    return out


def summarize(outcomes: list[RequestOutcome], wall_s: float | None = None) -> dict:
    good = [o for o in outcomes if o.ok]
    out: dict = {"completed_requests": len(good), "failed_requests": len(outcomes) - len(good)}
    if not good:
        return out
    out.update(_stats("latency", [o.latency_s for o in good], digits=3))
    for k in ("latency_mean", "latency_median", "latency_p95", "latency_p99"):
        if k in out:
            out[k + "_s"] = out.pop(k)
    ttfa = [o.ttfa_s for o in good if o.ttfa_s is not None]
    ttft = [o.ttft_s for o in good if o.ttft_s is not None]
    out.update({k + "_s": v for k, v in _stats("ttfa", ttfa, (50, 95), 4).items()})
    out.update({k + "_s": v for k, v in _stats("ttft", ttft, (50, 95), 4).items()})
    rtf = [o.rtf for o in good if o.rtf is not None]
    if rtf:
        out["rtf_mean"] = round(float(np.mean(rtf)), 4)
        out["rtf_median"] = round(float(np.median(rtf)), 4)
    audio = [o.audio_s for o in good if o.audio_s > 0]
    if audio:
        out["audio_duration_mean_s"] = round(float(np.mean(audio)), 3)
        if wall_s:
            out["audio_s_per_s"] = round(sum(audio) / wall_s, 3)
    busy = wall_s if wall_s and wall_s > 0 else sum(o.latency_s for o in good)
    out["throughput_qps"] = round(len(good) / busy, 3) if busy > 0 else 0.0
    rates = [o.tok_per_s for o in good if o.tok_per_s is not None]
    if rates:
        out["tok_per_s_mean"] = round(float(np.mean(rates)), 1)
        out["tok_per_s_median"] = round(float(np.median(rates)), 1)
    toks = sum(o.completion_tokens for o in good)
    eng = sum(o.engine_time_s for o in good if o.engine_time_s > 0)
    if toks and eng > 0:
        out["tok_per_s_agg"] = round(toks / eng, 1)
    if toks:
        out["gen_tokens_total"] = toks
    prompt = sum(o.prompt_tokens for o in good)
    if prompt:
        out["prompt_tokens_total"] = prompt
    return out


# metrics where larger is better; everything else listed in a baseline is latency-like
HIGHER_IS_BETTER = ("throughput_qps", "tok_per_s_agg", "tok_per_s_mean", "tok_per_s_median", "audio_s_per_s")


def regression_failures(summary: dict, baseline: dict, drop: float = 0.75, rise: float = 1.25) -> list[str]:
    """Metrics of ``summary`` that regress past the gate relative to ``baseline`` (a dict of
    the same keys, e.g. a P95 of earlier runs); missing metrics count as failures."""
    bad = []
    for k, ref in baseline.items():
        if ref is None:
            continue
        got = summary.get(k)
        if got is None:
            bad.append(f"{k}: missing (baseline {ref})")
        elif k in HIGHER_IS_BETTER and got < drop * ref:
            bad.append(f"{k}: {got} < {drop} x {ref}")
        elif k not in HIGHER_IS_BETTER and got > rise * ref:
            bad.append(f"{k}: {got} > {rise} x {ref}")
    return bad
