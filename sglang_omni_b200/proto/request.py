"""Request-level records shared by coordinator, stages and executors.

Same record shapes as the reference (sglang_omni/proto/request.py:9-82):
RequestState lifecycle PENDING -> RUNNING -> COMPLETED / FAILED / ABORTED,
OmniRequest (inputs + params + metadata), StagePayload (what travels between
stages).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import Any


class RequestState(Enum):
    PENDING = "pending"
    RUNNING = "running"
    COMPLETED = "completed"
    FAILED = "failed"
    ABORTED = "aborted"


@dataclass
class RequestInfo:
    request_id: str
    state: RequestState = RequestState.PENDING
    current_stage: str | None = None
    result: Any = None
    error: str | None = None


@dataclass
class OmniRequest:
    inputs: Any
    params: dict[str, Any] = field(default_factory=dict)
    metadata: dict[str, Any] = field(default_factory=dict)

    def to_dict(self) -> dict[str, Any]:
        return {"_type": "OmniRequest", "inputs": self.inputs, "params": self.params, "metadata": self.metadata}

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "OmniRequest":
        return cls(inputs=d.get("inputs"), params=d.get("params") or {}, metadata=d.get("metadata") or {})


@dataclass
class StagePayload:
    request_id: str
    request: OmniRequest
    data: Any = None

    def to_dict(self) -> dict[str, Any]:
        return {"_type": "StagePayload", "request_id": self.request_id, "request": self.request.to_dict(),
                "data": self.data}

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "StagePayload":
        req = d.get("request")
        if isinstance(req, dict):
            req = OmniRequest.from_dict(req)
        return cls(request_id=d["request_id"], request=req, data=d.get("data"))
