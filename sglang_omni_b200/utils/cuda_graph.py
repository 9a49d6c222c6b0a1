"""CUDA-graph capture that is safe while other threads of the process run GPU work.

Stages of one process (thinker, talker, vocoder, encoders) run their engines on
separate threads, and each captures its own graphs lazily, per batch bucket.
``torch.cuda.graph`` is not usable there: it captures in the "global" error
mode (any other thread's synchronous copy or allocation during the capture
then fails, and invalidates the capture), it synchronises the whole device and
empties the allocator cache on entry, and every graph shares one class-level
capture stream.  ``capture_graph`` instead warms the body up and captures it on
a private side stream in the "thread_local" mode, with stream-level syncs only.
Warm-up runs on the caller's stream, so it stays ordered with the rest of the
process's work on that stream.
"""
from __future__ import annotations

import threading
from typing import Any, Callable

import torch


_tls = threading.local()


def _capture_stream() -> torch.cuda.Stream:
    """One capture stream per thread (graphs captured by a thread share its per-stream scratch)."""
    s = getattr(_tls, "stream", None)
    if s is None or s.device != torch.device("cuda", torch.cuda.current_device()):
        s = _tls.stream = torch.cuda.Stream()
    return s


def capture_graph(body: Callable[[], Any], warmup: int = 2, pool=None) -> tuple[torch.cuda.CUDAGraph, Any]:
    """Run ``body`` ``warmup`` times, then capture one call of it.

    Returns (graph, outputs of the captured call).  The outputs are static:
    every ``graph.replay()`` rewrites them in place.
    """
    cur = torch.cuda.current_stream()
    # warm-up on the caller's stream: a side stream would run concurrently with
    # the work other threads keep queueing on that stream
    for _ in range(warmup):
        body()
    side = _capture_stream()
    with torch.cuda.stream(side):  # the stream's split-K scratch must exist before the capture starts
        from ..ops.gemm import splitk_scratch

        splitk_scratch(torch.device("cuda", torch.cuda.current_device()))
    side.wait_stream(cur)
    side.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        g.capture_begin(pool=pool, capture_error_mode="thread_local")
        try:
            out = body()
        except BaseException:
            try:
                g.capture_end()
            except Exception:
                pass
            raise
        g.capture_end()
    side.synchronize()
    cur.wait_stream(side)
    return g, out
