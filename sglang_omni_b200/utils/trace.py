"""Per-request event timestamps across pipeline stages (in-process pipelines).

With ``OMNI_TRACE=1`` the stages call :func:`mark` at fixed points of a
request's life (preprocessed, encoders done, first thinker token, first talker
frame, first audio chunk out); :func:`summary` gives, for every event, the
median delay after the request's first event.  Off by default: ``mark`` is then
a dictionary-free no-op.
"""
from __future__ import annotations

import os
import statistics
import threading
import time

ENABLED = os.environ.get("OMNI_TRACE", "0") not in ("", "0")
_lock = threading.Lock()
_events: dict[str, dict[str, float]] = {}
_batches: list[tuple[str, int, float]] = []


def mark(rid: str, event: str) -> None:
    """Records the first time `event` happens for request `rid`."""
    if not ENABLED:
        return
    t = time.perf_counter()
    with _lock:
        ev = _events.setdefault(rid, {})
        ev.setdefault(event, t)


def clear() -> None:
    with _lock:
        _events.clear()
        _batches.clear()


def summary(prefix: str = "") -> dict[str, float]:
    """Median milliseconds from each request's first mark to every event."""
    with _lock:
        items = [ev for rid, ev in _events.items() if rid.startswith(prefix) and ev]
    out: dict[str, list[float]] = {}
    for ev in items:
        t0 = min(ev.values())
        for k, v in ev.items():
            out.setdefault(k, []).append(1e3 * (v - t0))
    return {k: round(statistics.median(v), 2) for k, v in sorted(out.items(), key=lambda kv: statistics.median(kv[1]))}


def batch(stage: str, size: int, seconds: float) -> None:
    """Records one batched step of a stage (size, wall seconds)."""
    if ENABLED:
        with _lock:
            _batches.append((stage, size, seconds))


def batches() -> list[tuple[str, int, float]]:
    with _lock:
        return list(_batches)
