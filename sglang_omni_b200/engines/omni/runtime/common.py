"""Common runtime pieces: count-limited resources, single-pass and EOS /
max-length iteration controllers (sglang_omni/engines/omni/runtime/common.py)."""
from __future__ import annotations

from ..types import SchedulerRequest


class SimpleResourceManager:
    def __init__(self, max_count: int = 64):
        self.max_count = max_count
        self.in_use = 0

    def can_allocate(self, request: SchedulerRequest) -> bool:
        return self.in_use < self.max_count

    def allocate(self, request: SchedulerRequest) -> None:
        self.in_use += 1

    def free(self, request: SchedulerRequest) -> None:
        self.in_use = max(0, self.in_use - 1)


class SinglePassIterationController:
    def update_request(self, request, output):
        request.data = output if output is not None else request.data

    def is_finished(self, request, output) -> bool:
        return True


class EosIterationController:
    def __init__(self, eos_token_ids=(), max_new_tokens: int = 128, max_length: int | None = None):
        self.eos = set(eos_token_ids)
        self.max_new_tokens = max_new_tokens
        self.max_length = max_length

    def update_request(self, request, output):
        request.data.setdefault("output_ids", []).append(int(output))

    def is_finished(self, request, output) -> bool:
        out = request.data.get("output_ids", [])
        if out and out[-1] in self.eos:
            return True
        if len(out) >= request.data.get("max_new_tokens", self.max_new_tokens):
            return True
        if self.max_length is not None and len(request.data.get("input_ids", [])) + len(out) >= self.max_length:
            return True
        return False
