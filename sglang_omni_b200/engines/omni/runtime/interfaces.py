"""Pluggable pieces of the generic step engine (sglang_omni/engines/omni/runtime/interfaces.py:13-97)."""
from __future__ import annotations

from typing import Any, Protocol

from ..types import ModelRunnerOutput, SchedulerOutput, SchedulerRequest


class BatchPlanner(Protocol):
    def select_requests(self, waiting: list[SchedulerRequest], running: list[SchedulerRequest],
                        resources: "ResourceManager") -> list[SchedulerRequest]: ...

    def build_batch(self, requests: list[SchedulerRequest]) -> Any: ...


class ResourceManager(Protocol):
    def can_allocate(self, request: SchedulerRequest) -> bool: ...

    def allocate(self, request: SchedulerRequest) -> None: ...

    def free(self, request: SchedulerRequest) -> None: ...


class IterationController(Protocol):
    def update_request(self, request: SchedulerRequest, output: Any) -> None: ...

    def is_finished(self, request: SchedulerRequest, output: Any) -> bool: ...


class InputPreparer(Protocol):
    def prepare(self, scheduler_output: SchedulerOutput, device) -> dict[str, Any]: ...


class OutputProcessor(Protocol):
    def process(self, model_output: Any, scheduler_output: SchedulerOutput) -> ModelRunnerOutput: ...


class CacheManager(Protocol):
    def get(self, request: SchedulerRequest) -> Any | None: ...

    def put(self, request: SchedulerRequest, output: Any) -> None: ...
