"""Request driver: warm-up requests one at a time, then every sample with at most
``concurrency`` requests in flight, optionally released at a Poisson ``rate`` (requests per
second; inf releases them all at once), as the reference's BenchmarkRunner
(benchmarks/benchmarker/runner.py:30-110) does."""
from __future__ import annotations

import asyncio
import math
import random
import time
from typing import Awaitable, Callable, Sequence

from .results import RequestOutcome

Send = Callable[[object, int], Awaitable[RequestOutcome]]   # (sample, index) -> outcome


async def run_requests(samples: Sequence, send: Send, concurrency: int = 1, rate: float = math.inf,
                       warmup: int = 1, seed: int = 0,
                       progress: Callable[[int, int], None] | None = None) -> tuple[list[RequestOutcome], float]:
    """Returns (outcomes in sample order, wall seconds of the measured part)."""
    for i in range(min(warmup, len(samples))):
        await send(samples[i], -1 - i)
    gate = asyncio.Semaphore(max(1, concurrency))
    done = 0
    rnd = random.Random(seed)

    async def one(i: int, sample) -> RequestOutcome:
        nonlocal done
        async with gate:
            try:
                res = await send(sample, i)
            except Exception as exc:      # a failed request is an outcome, not a crash
                res = RequestOutcome(request_id=str(i), error=f"{type(exc).__name__}: {exc}")
        done += 1
        if progress is not None:
            progress(done, len(samples))
        return res

    t0 = time.perf_counter()
    tasks = []
    for i, sample in enumerate(samples):
        if math.isfinite(rate) and rate > 0 and i:
            await asyncio.sleep(rnd.expovariate(rate))
        tasks.append(asyncio.ensure_future(one(i, sample)))
    out = list(await asyncio.gather(*tasks))
    return out, time.perf_counter() - t0
