"""Stage input handlers: direct pass-through, or aggregated fan-in that waits for
every source stage and merges their payloads in source order
(sglang_omni/pipeline/stage/input.py:14-119)."""
from __future__ import annotations

from typing import Callable

from ...proto import StagePayload


class InputHandler:
    def receive(self, request_id: str, from_stage: str | None, payload: StagePayload) -> StagePayload | None:
        raise NotImplementedError

    def cancel(self, request_id: str) -> None:
        pass


class DirectInput(InputHandler):
    def receive(self, request_id, from_stage, payload):
        return payload


class AggregatedInput(InputHandler):
    def __init__(self, sources: list[str], merge: Callable[[dict[str, StagePayload]], StagePayload] | None = None):
        self.sources = list(sources)
        self.merge = merge
        self._pending: dict[str, dict[str, StagePayload]] = {}

    def receive(self, request_id, from_stage, payload):
        got = self._pending.setdefault(request_id, {})
        key = from_stage if from_stage in self.sources else f"_{len(got)}"
        got[key] = payload
        if not all(s in got for s in self.sources):
            return None
        del self._pending[request_id]
        ordered = {s: got[s] for s in self.sources}
        if self.merge is not None:
            return self.merge(ordered)
        first = ordered[self.sources[0]]
        return StagePayload(request_id=request_id, request=first.request,
                            data={s: p.data for s, p in ordered.items()})

    def cancel(self, request_id):
        self._pending.pop(request_id, None)
