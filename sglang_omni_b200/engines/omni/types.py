"""Scheduler-side request records (sglang_omni/engines/omni/types.py:9-87)."""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from enum import Enum
from typing import Any


class SchedulerStatus(Enum):
    WAITING = "waiting"
    RUNNING = "running"
    WAITING_FEEDBACK = "waiting_feedback"
    FINISHED = "finished"
    ABORTED = "aborted"


@dataclass
class SchedulerRequest:
    request_id: str
    data: Any
    status: SchedulerStatus = SchedulerStatus.WAITING
    arrival: float = field(default_factory=time.perf_counter)
    finish_time: float | None = None
    error: str | None = None
    num_steps: int = 0


@dataclass
class SchedulerOutput:
    requests: list[SchedulerRequest]
    batch_data: Any = None
    step_id: int = 0


@dataclass
class RequestOutput:
    request_id: str
    data: Any = None
    finished: bool = False
    extra: dict[str, Any] = field(default_factory=dict)


@dataclass
class ModelRunnerOutput:
    outputs: dict[str, RequestOutput]
    req_ids: list[str] = field(default_factory=list)
