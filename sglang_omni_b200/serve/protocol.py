"""OpenAI-compatible request / response models with the omni extensions.
Field names match sglang_omni/serve/protocol.py:15-230 (images / audios /
videos / modalities / audio / stage_sampling / stage_params / request_id;
speech: references, ref_audio, task_type, ...)."""
from __future__ import annotations

import time
from typing import Any

from pydantic import BaseModel, Field


class UsageResponse(BaseModel):
    prompt_tokens: int = 0
    completion_tokens: int = 0
    total_tokens: int = 0
    engine_time_s: float | None = None


class ChatMessage(BaseModel):
    role: str
    content: Any = None
    name: str | None = None
    tool_calls: list[dict[str, Any]] | None = None
    tool_call_id: str | None = None


class ChatCompletionAudio(BaseModel):
    id: str
    data: str
    expires_at: int | None = None
    transcript: str | None = None


class ChatCompletionRequest(BaseModel):
    model: str | None = None
    messages: list[ChatMessage]
    temperature: float | None = None
    top_p: float | None = None
    top_k: int | None = None
    min_p: float | None = None
    repetition_penalty: float | None = None
    max_tokens: int | None = None
    max_completion_tokens: int | None = None
    stop: str | list[str] | None = None
    seed: int | None = None
    stream: bool = False
    modalities: list[str] | None = None
    audio: dict[str, Any] | None = None
    audios: list[str] | None = None
    images: list[str] | None = None
    videos: list[str] | None = None
    stage_sampling: dict[str, dict[str, Any]] | None = None
    stage_params: dict[str, dict[str, Any]] | None = None
    request_id: str | None = None
    user: str | None = None
    ignore_eos: bool | None = None
    prompt_token_ids: list[int] | None = None


class ChatCompletionChoice(BaseModel):
    index: int = 0
    message: dict[str, Any]
    finish_reason: str | None = "stop"


class ChatCompletionResponse(BaseModel):
    id: str
    object: str = "chat.completion"
    created: int = Field(default_factory=lambda: int(time.time()))
    model: str
    choices: list[ChatCompletionChoice]
    usage: UsageResponse | None = None


class ChatCompletionStreamDelta(BaseModel):
    role: str | None = None
    content: str | None = None
    audio: ChatCompletionAudio | None = None


class ChatCompletionStreamChoice(BaseModel):
    index: int = 0
    delta: ChatCompletionStreamDelta
    finish_reason: str | None = None


class ChatCompletionStreamResponse(BaseModel):
    id: str
    object: str = "chat.completion.chunk"
    created: int = Field(default_factory=lambda: int(time.time()))
    model: str
    choices: list[ChatCompletionStreamChoice]
    usage: UsageResponse | None = None


class SpeechReference(BaseModel):
    audio_path: str | None = None
    text: str | None = None
    vq_codes: list[list[int]] | list[int] | None = None


class CreateSpeechRequest(BaseModel):
    model: str | None = None
    input: str
    voice: str = "default"
    response_format: str = "wav"
    speed: float = 1.0
    stream: bool = False
    task_type: str | None = None
    language: str | None = None
    instructions: str | None = None
    ref_audio: str | None = None
    ref_text: str | None = None
    references: list[SpeechReference] | None = None
    max_new_tokens: int | None = None
    temperature: float | None = None
    top_p: float | None = None
    top_k: int | None = None
    repetition_penalty: float | None = None
    seed: int | None = None
    stage_params: dict[str, dict[str, Any]] | None = None


class ModelPermission(BaseModel):
    id: str = "modelperm-default"
    object: str = "model_permission"
    allow_create_engine: bool = False
    allow_sampling: bool = True
    allow_logprobs: bool = True


class ModelCard(BaseModel):
    id: str
    object: str = "model"
    created: int = 0
    owned_by: str = "sglang-omni-b200"
    permission: list[ModelPermission] = Field(default_factory=lambda: [ModelPermission()])
    root: str | None = None


class ModelList(BaseModel):
    object: str = "list"
    data: list[ModelCard] = Field(default_factory=list)
