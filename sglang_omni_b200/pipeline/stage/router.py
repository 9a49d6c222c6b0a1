"""Round-robin worker routing with sticky per-request affinity, so a request
that re-enters a stage (streaming chunks, feedback) lands on the worker that
holds its KV state (sglang_omni/pipeline/stage/router.py:11-47)."""
from __future__ import annotations


class WorkerRouter:
    def __init__(self, num_workers: int):
        self.num_workers = max(1, num_workers)
        self._next = 0
        self._affinity: dict[str, int] = {}

    def route(self, request_id: str) -> int:
        w = self._affinity.get(request_id)
        if w is None:
            w = self._next
            self._next = (self._next + 1) % self.num_workers
            self._affinity[request_id] = w
        return w

    def release(self, request_id: str) -> None:
        self._affinity.pop(request_id, None)
