"""Control-plane messages.

Every message has ``to_dict`` / ``from_dict`` with a ``type`` discriminator and
is msgpack-serialisable; tensors never travel here (they go through a relay and
the message carries the relay metadata).  Message set and fields follow the
reference (sglang_omni/proto/messages.py:11-306): data_ready (with chunk_id /
is_done / error for streaming), submit, complete, stream, abort, shutdown,
profiler_start, profiler_stop.
"""
from __future__ import annotations

import base64
import pickle
from dataclasses import dataclass
from typing import Any

from .request import StagePayload


def _pack_obj(obj: Any) -> Any:
    """Encodes arbitrary (picklable, tensor-free) Python data for msgpack."""
    if obj is None or isinstance(obj, (bool, int, float, str, bytes)):
        return obj
    return {"__pickled__": base64.b64encode(pickle.dumps(obj, protocol=pickle.HIGHEST_PROTOCOL)).decode()}


def _unpack_obj(obj: Any) -> Any:
    if isinstance(obj, dict) and "__pickled__" in obj:
        return pickle.loads(base64.b64decode(obj["__pickled__"]))
    return obj


@dataclass
class DataReadyMessage:
    request_id: str
    from_stage: str
    to_stage: str
    shm_metadata: Any           # relay metadata (dict) or an inline payload marker
    chunk_id: int | None = None
    is_done: bool = False
    error: str | None = None

    def to_dict(self) -> dict[str, Any]:
        d = {"type": "data_ready", "request_id": self.request_id, "from_stage": self.from_stage,
             "to_stage": self.to_stage, "shm_metadata": _pack_obj(self.shm_metadata)}
        if self.chunk_id is not None:
            d["chunk_id"] = self.chunk_id
        if self.is_done:
            d["is_done"] = True
        if self.error is not None:
            d["error"] = self.error
        return d

    @classmethod
    def from_dict(cls, d):
        return cls(d["request_id"], d["from_stage"], d["to_stage"], _unpack_obj(d.get("shm_metadata")),
                   d.get("chunk_id"), bool(d.get("is_done", False)), d.get("error"))


@dataclass
class AbortMessage:
    request_id: str

    def to_dict(self):
        return {"type": "abort", "request_id": self.request_id}

    @classmethod
    def from_dict(cls, d):
        return cls(d["request_id"])


@dataclass
class CompleteMessage:
    request_id: str
    from_stage: str
    success: bool
    result: Any = None
    error: str | None = None

    def to_dict(self):
        return {"type": "complete", "request_id": self.request_id, "from_stage": self.from_stage,
                "success": self.success, "result": _pack_obj(self.result), "error": self.error}

    @classmethod
    def from_dict(cls, d):
        return cls(d["request_id"], d["from_stage"], bool(d["success"]), _unpack_obj(d.get("result")), d.get("error"))


@dataclass
class StreamMessage:
    request_id: str
    from_stage: str
    chunk: Any
    stage_id: int | None = None
    stage_name: str | None = None
    modality: str | None = None
    seq: int | None = None      # per (request, stage) chunk number: duplicates are dropped

    def to_dict(self):
        d = {"type": "stream", "request_id": self.request_id, "from_stage": self.from_stage,
             "chunk": _pack_obj(self.chunk), "stage_id": self.stage_id, "stage_name": self.stage_name,
             "modality": self.modality}
        if self.seq is not None:
            d["seq"] = self.seq
        return d

    @classmethod
    def from_dict(cls, d):
        return cls(d["request_id"], d["from_stage"], _unpack_obj(d.get("chunk")), d.get("stage_id"),
                   d.get("stage_name"), d.get("modality"), d.get("seq"))


@dataclass
class SubmitMessage:
    request_id: str
    data: Any

    def to_dict(self):
        data = self.data.to_dict() if isinstance(self.data, StagePayload) else self.data
        return {"type": "submit", "request_id": self.request_id, "data": _pack_obj(data)}

    @classmethod
    def from_dict(cls, d):
        data = _unpack_obj(d.get("data"))
        if isinstance(data, dict) and data.get("_type") == "StagePayload":
            data = StagePayload.from_dict(data)
        return cls(d["request_id"], data)


@dataclass
class ShutdownMessage:
    def to_dict(self):
        return {"type": "shutdown"}

    @classmethod
    def from_dict(cls, d):
        return cls()


@dataclass
class ProfilerStartMessage:
    run_id: str
    trace_path_template: str

    def to_dict(self):
        return {"type": "profiler_start", "run_id": self.run_id, "trace_path_template": self.trace_path_template}

    @classmethod
    def from_dict(cls, d):
        return cls(d["run_id"], d["trace_path_template"])


@dataclass
class ProfilerStopMessage:
    run_id: str

    def to_dict(self):
        return {"type": "profiler_stop", "run_id": self.run_id}

    @classmethod
    def from_dict(cls, d):
        return cls(d["run_id"])


@dataclass
class StageStatsMessage:
    """Periodic load report of a stage to the coordinator (queue depth, engine state)."""
    stage: str
    stats: dict

    def to_dict(self):
        return {"type": "stage_stats", "stage": self.stage, "stats": self.stats}

    @classmethod
    def from_dict(cls, d):
        return cls(d["stage"], dict(d.get("stats") or {}))


_TYPES = {
    "data_ready": DataReadyMessage, "abort": AbortMessage, "complete": CompleteMessage, "stream": StreamMessage,
    "submit": SubmitMessage, "shutdown": ShutdownMessage, "profiler_start": ProfilerStartMessage,
    "profiler_stop": ProfilerStopMessage, "stage_stats": StageStatsMessage,
}


def parse_message(d: dict[str, Any]):
    t = d.get("type")
    cls = _TYPES.get(t)
    if cls is None:
        raise ValueError(f"unknown message type: {t!r}")
    return cls.from_dict(d)
