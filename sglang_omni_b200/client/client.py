"""In-process client over a Coordinator: builds OmniRequests from
GenerateRequests, streams GenerateChunks, aggregates text and audio, merges
multi-terminal results ({"decode": ..., "code2wav": ...}), encodes audio.

Reference counterpart: sglang_omni/client/client.py:33-432.
"""
from __future__ import annotations

import base64
import time
import uuid
from typing import Any, AsyncIterator

import numpy as np

from ..pipeline.coordinator import Coordinator
from ..proto import OmniRequest, StreamMessage
from .audio import encode_audio
from .types import (AbortLevel, AbortResult, CompletionAudio, CompletionResult, CompletionStreamChunk,
                    GenerateChunk, GenerateRequest, SpeechResult, UsageInfo)


def _usage_of(res: Any) -> UsageInfo | None:
    if isinstance(res, dict):
        u = res.get("usage")
        if isinstance(u, dict):
            return UsageInfo(u.get("prompt_tokens"), u.get("completion_tokens"), u.get("total_tokens"),
                             u.get("engine_time_s"))
        for v in res.values():
            if isinstance(v, dict) and isinstance(v.get("usage"), dict):
                return _usage_of(v)
    return None


def _text_of(res: Any) -> str:
    if isinstance(res, dict):
        if isinstance(res.get("text"), str):
            return res["text"]
        for k in ("decode", "thinker", "tts_engine"):
            if isinstance(res.get(k), dict) and isinstance(res[k].get("text"), str):
                return res[k]["text"]
    if isinstance(res, str):
        return res
    return ""


def _audio_of(res: Any):
    """Returns (float32 waveform, sample rate) from a (multi-terminal) result, if any."""
    if isinstance(res, dict):
        if "audio_waveform" in res:
            w = res["audio_waveform"]
            if isinstance(w, (bytes, bytearray)):
                w = np.frombuffer(w, dtype=np.float32)
            elif hasattr(w, "detach"):
                w = w.detach().float().cpu().numpy()
            return np.asarray(w, dtype=np.float32).reshape(-1), int(res.get("sample_rate", 24000))
        for k in ("code2wav", "vocoder", "talker"):
            if k in res:
                a = _audio_of(res[k])
                if a is not None:
                    return a
    return None


class Client:
    def __init__(self, coordinator: Coordinator, tokenizer=None, model_name: str = "model"):
        self.coordinator = coordinator
        self.tokenizer = tokenizer
        self.model_name = model_name

    # ------------------------------------------------------------------ request building
    def _build_params(self, req: GenerateRequest) -> dict[str, Any]:
        sampling = req.sampling.to_dict()
        if req.max_tokens is not None:
            sampling["max_new_tokens"] = req.max_tokens
        params: dict[str, Any] = {"sampling": sampling, "stream": bool(req.stream)}
        if req.stage_sampling:
            params["stage_sampling"] = {k: (v.to_dict() if hasattr(v, "to_dict") else dict(v))
                                        for k, v in req.stage_sampling.items()}
        if req.stage_params:
            params["stage_params"] = req.stage_params
        if req.output_modalities:
            params["output_modalities"] = list(req.output_modalities)
        if req.task:
            params["task"] = req.task
        return params

    def _extract_inputs(self, req: GenerateRequest) -> dict[str, Any]:
        inputs: dict[str, Any] = {}
        if req.prompt_token_ids is not None:
            inputs["prompt_token_ids"] = list(req.prompt_token_ids)
        if req.prompt is not None:
            inputs["prompt"] = req.prompt
        if req.messages is not None:
            inputs["messages"] = [m if isinstance(m, dict) else {"role": m.role, "content": m.content}
                                  for m in req.messages]
        for k in ("images", "audios", "videos"):
            v = getattr(req, k)
            if v:
                inputs[k] = list(v)
        return inputs

    def _omni_request(self, req: GenerateRequest) -> tuple[str, OmniRequest]:
        rid = req.request_id or f"req-{uuid.uuid4().hex[:16]}"
        meta = dict(req.metadata)
        meta["submitted_at"] = time.time()
        return rid, OmniRequest(inputs=self._extract_inputs(req), params=self._build_params(req), metadata=meta)

    # ------------------------------------------------------------------ generation
    async def generate(self, req: GenerateRequest) -> AsyncIterator[GenerateChunk]:
        rid, oreq = self._omni_request(req)
        if not req.stream:
            res = await self.coordinator.submit(rid, oreq)
            yield self._final_chunk(rid, res)
            return
        idx = 0
        async for item in self.coordinator.stream(rid, oreq):
            if isinstance(item, StreamMessage):
                ch = item.chunk if isinstance(item.chunk, dict) else {"text": str(item.chunk)}
                modality = ch.get("modality") or item.modality or "text"
                audio = ch.get("audio_waveform")
                yield GenerateChunk(request_id=rid, index=idx, token_ids=list(ch.get("token_ids") or []),
                                    text=ch.get("text", "") or "", stage_id=item.stage_id,
                                    stage_name=item.stage_name, modality=modality, audio_data=audio,
                                    sample_rate=ch.get("sample_rate"))
                idx += 1
            else:
                yield self._final_chunk(rid, item["result"], idx)

    def _final_chunk(self, rid: str, res: Any, idx: int = 0) -> GenerateChunk:
        finish = "stop"
        if isinstance(res, dict):
            finish = res.get("finish_reason") or (res.get("decode") or {}).get("finish_reason") or "stop"
        audio = _audio_of(res)
        return GenerateChunk(request_id=rid, index=idx, text=_text_of(res), finish_reason=finish,
                             usage=_usage_of(res), modality="audio" if audio is not None else "text",
                             audio_data=None if audio is None else audio[0],
                             sample_rate=None if audio is None else audio[1],
                             token_ids=list(res.get("token_ids") or []) if isinstance(res, dict) else [])

    async def completion(self, req: GenerateRequest) -> CompletionResult:
        req.stream = False
        final = None
        async for ch in self.generate(req):
            final = ch
        audio = None
        if final.audio_data is not None:
            wav = encode_audio(final.audio_data, final.sample_rate or 24000, "wav")
            audio = CompletionAudio(id=f"audio-{final.request_id}", data=base64.b64encode(wav).decode())
        return CompletionResult(request_id=final.request_id, text=final.text, audio=audio,
                                finish_reason=final.finish_reason or "stop", usage=final.usage,
                                token_ids=final.token_ids)

    async def completion_stream(self, req: GenerateRequest) -> AsyncIterator[CompletionStreamChunk]:
        req.stream = True
        async for ch in self.generate(req):
            if ch.finish_reason is not None:
                yield CompletionStreamChunk(ch.request_id, "", "text", None, ch.finish_reason, ch.usage,
                                            ch.stage_name)
                continue
            if ch.modality == "audio" and ch.audio_data is not None:
                data = ch.audio_data
                if isinstance(data, (bytes, bytearray)):
                    data = np.frombuffer(data, dtype=np.float32)
                wav = encode_audio(np.asarray(data, dtype=np.float32), ch.sample_rate or 24000, "wav")
                yield CompletionStreamChunk(ch.request_id, "", "audio", base64.b64encode(wav).decode(), None, None,
                                            ch.stage_name)
            elif ch.text:
                yield CompletionStreamChunk(ch.request_id, ch.text, "text", None, None, None, ch.stage_name)

    async def speech(self, req: GenerateRequest, response_format: str = "wav") -> SpeechResult:
        req.stream = False
        req.task = req.task or "tts"
        final = None
        async for ch in self.generate(req):
            final = ch
        if final is None or final.audio_data is None:
            raise RuntimeError("pipeline returned no audio")
        data, fmt, mime = encode_audio(final.audio_data, final.sample_rate or 24000, response_format,
                                       return_meta=True)
        return SpeechResult(audio_bytes=data, mime_type=mime, format=fmt, usage=final.usage)

    async def abort(self, request_id: str, level: AbortLevel = AbortLevel.SOFT) -> AbortResult:
        ok = await self.coordinator.abort(request_id)
        return AbortResult(success=ok, level_applied=level)

    def get_status(self) -> dict:
        return self.coordinator.health()

    def health(self) -> bool:
        return bool(self.coordinator.running)
