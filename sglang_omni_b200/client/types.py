"""Client-side request / chunk / result types (field names as in
sglang_omni/client/types.py:11-222)."""
from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import Any

from ..sampling_params import SamplingParams


@dataclass
class Message:
    role: str
    content: Any


@dataclass
class UsageInfo:
    prompt_tokens: int | None = None
    completion_tokens: int | None = None
    total_tokens: int | None = None
    engine_time_s: float | None = None

    def to_dict(self) -> dict[str, Any]:
        return {k: v for k, v in self.__dict__.items() if v is not None}


@dataclass
class GenerateRequest:
    model: str | None = None
    prompt: str | None = None
    prompt_token_ids: list[int] | None = None
    messages: list[Message] | None = None
    images: list[Any] | None = None
    audios: list[Any] | None = None
    videos: list[Any] | None = None
    sampling: SamplingParams = field(default_factory=SamplingParams)
    stage_sampling: dict[str, SamplingParams] | None = None
    stage_params: dict[str, dict[str, Any]] | None = None
    stream: bool = True
    max_tokens: int | None = None
    output_modalities: list[str] | None = None
    task: str | None = None
    request_id: str | None = None
    metadata: dict[str, Any] = field(default_factory=dict)


@dataclass
class GenerateChunk:
    request_id: str
    index: int = 0
    token_ids: list[int] = field(default_factory=list)
    text: str = ""
    logprobs: list[float] | None = None
    finish_reason: str | None = None
    usage: UsageInfo | None = None
    stage_id: int | None = None
    stage_name: str | None = None
    modality: str = "text"
    audio_data: Any = None
    sample_rate: int | None = None


class AbortLevel(Enum):
    SOFT = "soft"
    HARD = "hard"


@dataclass
class AbortResult:
    success: bool
    level_applied: AbortLevel
    partial_output: GenerateChunk | None = None


@dataclass
class CompletionAudio:
    id: str
    data: str
    transcript: str | None = None


@dataclass
class CompletionResult:
    request_id: str
    text: str
    audio: CompletionAudio | None = None
    finish_reason: str = "stop"
    usage: UsageInfo | None = None
    token_ids: list[int] | None = None


@dataclass
class CompletionStreamChunk:
    request_id: str
    text: str = ""
    modality: str = "text"
    audio_b64: str | None = None
    finish_reason: str | None = None
    usage: UsageInfo | None = None
    stage_name: str | None = None


@dataclass
class SpeechResult:
    audio_bytes: bytes
    mime_type: str
    format: str
    usage: UsageInfo | None = None


class ClientError(Exception):
    pass
