"""Server-side request metrics served at /metrics: counts, latency and
time-to-first-audio-chunk percentiles, output tokens."""
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
        self.lat = deque(maxlen=window)
        self.ttfa = deque(maxlen=window)

    def finished(self, latency_s: float, ttfa_s: float | None, tokens: int | None):
        with self._lock:
            self.ok += 1
            self.tokens += int(tokens or 0)
            self.lat.append(latency_s)
            if ttfa_s is not None:
                self.ttfa.append(ttfa_s)

    def failed(self):
        with self._lock:
            self.err += 1

    def snapshot(self) -> dict:
        with self._lock:
            lat, ttfa = list(self.lat), list(self.ttfa)
            return {"requests_ok": self.ok, "requests_failed": self.err, "completion_tokens": self.tokens,
                    "latency_p50_s": _pct(lat, 0.5), "latency_p99_s": _pct(lat, 0.99),
                    "ttfa_p50_s": _pct(ttfa, 0.5), "ttfa_p99_s": _pct(ttfa, 0.99)}
