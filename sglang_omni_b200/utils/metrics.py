"""Server-side request metrics served at /metrics (JSON, or the Prometheus text format with
``?format=prometheus``): request counts, requests in flight, completion tokens, and p50 / p99 of
request latency, time to first token, inter-token latency and time to first audio chunk."""
from __future__ import annotations

import threading
from collections import deque


def _pct(xs, q):
    if not xs:
        return None
    s = sorted(xs)
    i = min(len(s) - 1, max(0, int(round(q * (len(s) - 1)))))
    return s[i]


class ServerMetrics:
    def __init__(self, window: int = 4096):
        self._lock = threading.Lock()
        self.ok = 0
        self.err = 0
        self.tokens = 0
        self.in_flight = 0
        self.lat = deque(maxlen=window)
        self.ttft = deque(maxlen=window)
        self.itl = deque(maxlen=window)
        self.ttfa = deque(maxlen=window)

    def started(self):
        with self._lock:
            self.in_flight += 1

    def finished(self, latency_s: float, ttfa_s: float | None, tokens: int | None, ttft_s: float | None = None,
                 itl_s: float | None = None):
        with self._lock:
            self.ok += 1
            self.in_flight = max(0, self.in_flight - 1)
            self.tokens += int(tokens or 0)
            self.lat.append(latency_s)
            if ttfa_s is not None:
                self.ttfa.append(ttfa_s)
            if ttft_s is not None:
                self.ttft.append(ttft_s)
            if itl_s is not None:
                self.itl.append(itl_s)

    def failed(self):
        with self._lock:
            self.err += 1
            self.in_flight = max(0, self.in_flight - 1)

    def snapshot(self) -> dict:
        with self._lock:
            lat, ttfa, ttft, itl = list(self.lat), list(self.ttfa), list(self.ttft), list(self.itl)
            return {"requests_ok": self.ok, "requests_failed": self.err, "requests_in_flight": self.in_flight,
                    "completion_tokens": self.tokens,
                    "latency_p50_s": _pct(lat, 0.5), "latency_p99_s": _pct(lat, 0.99),
                    "ttft_p50_s": _pct(ttft, 0.5), "ttft_p99_s": _pct(ttft, 0.99),
                    "itl_p50_s": _pct(itl, 0.5), "itl_p99_s": _pct(itl, 0.99),
                    "ttfa_p50_s": _pct(ttfa, 0.5), "ttfa_p99_s": _pct(ttfa, 0.99)}

    def prometheus(self, prefix: str = "omni") -> str:
        """The snapshot in the Prometheus text exposition format (counters, a gauge and
        quantile series of summaries)."""
        s = self.snapshot()
        out = [f"# TYPE {prefix}_requests_total counter",
               f'{prefix}_requests_total{{status="ok"}} {s["requests_ok"]}',
               f'{prefix}_requests_total{{status="failed"}} {s["requests_failed"]}',
               f"# TYPE {prefix}_completion_tokens_total counter",
               f"{prefix}_completion_tokens_total {s['completion_tokens']}",
               f"# TYPE {prefix}_requests_in_flight gauge",
               f"{prefix}_requests_in_flight {s['requests_in_flight']}"]
        for name, key in (("request_latency_seconds", "latency"), ("time_to_first_token_seconds", "ttft"),
                          ("inter_token_latency_seconds", "itl"), ("time_to_first_audio_seconds", "ttfa")):
            out.append(f"# TYPE {prefix}_{name} summary")
            for q, label in (("50", "0.5"), ("99", "0.99")):
                v = s[f"{key}_p{q}_s"]
                if v is not None:
                    out.append(f'{prefix}_{name}{{quantile="{label}"}} {v:.6f}')
        return "\n".join(out) + "\n"
