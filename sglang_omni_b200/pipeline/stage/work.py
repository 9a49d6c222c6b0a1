"""Units of work handed from a stage to its workers (sglang_omni/pipeline/stage/work.py)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

from ...proto import StagePayload


@dataclass
class InputRef:
    """Exactly one of an inline payload or relay metadata."""

    payload: StagePayload | None = None
    metadata: Any = None

    def __post_init__(self):
        if (self.payload is None) == (self.metadata is None):
            raise ValueError("InputRef needs exactly one of payload / metadata")


@dataclass
class WorkDescriptor:
    request_id: str
    payload: StagePayload
    from_stage: str | None = None
