"""OpenAI-compatible FastAPI app.

Routes (same contract as sglang_omni/serve/openai_api.py:57-632):
  POST /v1/chat/completions   non-stream JSON, or SSE: role chunk, text / audio
                              deltas, a finish chunk with usage, ``[DONE]``
  POST /v1/audio/speech       raw audio bytes with X-Prompt-Tokens /
                              X-Completion-Tokens / X-Engine-Time headers, or
                              SSE ``audio.speech.chunk`` objects (``audio.data``
                              base64), a closing one with usage, ``[DONE]``
  GET  /v1/models, GET /health (503 when the coordinator is not running)
  GET  /metrics               request counters and latency percentiles
"""
from __future__ import annotations

import base64
import json
import time
import uuid
from typing import Any

import numpy as np
from fastapi import FastAPI, HTTPException
from fastapi.responses import JSONResponse, Response, StreamingResponse

from ..client import Client, GenerateRequest, Message, SamplingParams
from ..client.audio import encode_audio
from ..utils.metrics import ServerMetrics
from .protocol import (ChatCompletionAudio, ChatCompletionChoice, ChatCompletionRequest, ChatCompletionResponse,
                       ChatCompletionStreamChoice, ChatCompletionStreamDelta, ChatCompletionStreamResponse,
                       CreateSpeechRequest, ModelCard, ModelList, UsageResponse)

# S2-Pro style TTS sampling defaults (sglang_omni/serve/openai_api.py:589-591)
SPEECH_DEFAULTS = {"temperature": 0.8, "top_p": 0.8, "top_k": 30, "repetition_penalty": 1.1}


def _sse(obj: Any) -> str:
    if hasattr(obj, "model_dump"):
        obj = obj.model_dump(exclude_none=True)
    return f"data: {json.dumps(obj)}\n\n"


def build_chat_generate_request(req: ChatCompletionRequest) -> GenerateRequest:
    sp = SamplingParams()
    for k in ("temperature", "top_p", "top_k", "min_p", "repetition_penalty", "seed"):
        v = getattr(req, k)
        if v is not None:
            setattr(sp, k, v)
    if req.stop:
        sp.stop = [req.stop] if isinstance(req.stop, str) else list(req.stop)
    if req.ignore_eos:
        sp.ignore_eos = True
    max_tokens = req.max_completion_tokens or req.max_tokens
    if max_tokens is not None:
        sp.max_new_tokens = max_tokens
    stage_sampling = None
    if req.stage_sampling:
        stage_sampling = {k: SamplingParams.from_dict(v) for k, v in req.stage_sampling.items()}
    msgs = [Message(role=m.role, content=m.content) for m in req.messages]
    modalities = req.modalities or ["text"]
    return GenerateRequest(model=req.model, messages=msgs, prompt_token_ids=req.prompt_token_ids,
                           images=req.images, audios=req.audios, videos=req.videos, sampling=sp,
                           stage_sampling=stage_sampling, stage_params=req.stage_params, stream=req.stream,
                           max_tokens=max_tokens, output_modalities=modalities, request_id=req.request_id,
                           metadata={"audio": req.audio or {}})


def build_speech_generate_request(req: CreateSpeechRequest) -> GenerateRequest:
    sp = SamplingParams(**SPEECH_DEFAULTS)
    for k in ("temperature", "top_p", "top_k", "repetition_penalty", "seed"):
        v = getattr(req, k)
        if v is not None:
            setattr(sp, k, v)
    if req.max_new_tokens is not None:
        sp.max_new_tokens = req.max_new_tokens
    params = dict(req.stage_params or {})
    refs = [r.model_dump() for r in (req.references or [])]
    if req.ref_audio:
        refs.append({"audio_path": req.ref_audio, "text": req.ref_text})
    return GenerateRequest(model=req.model, prompt=req.input, sampling=sp, stage_params=params, stream=req.stream,
                           output_modalities=["audio"], task="tts",
                           metadata={"voice": req.voice, "speed": req.speed, "references": refs,
                                     "task_type": req.task_type, "language": req.language,
                                     "instructions": req.instructions, "response_format": req.response_format})


def stage_prometheus(stages: dict, prefix: str = "omni_stage") -> str:
    """Gauges ``omni_stage_<field>{stage="<name>"}`` of the numeric fields of the stage reports."""
    fields: dict[str, list[str]] = {}
    for name, st in sorted(stages.items()):
        for k, v in sorted(st.items()):
            if isinstance(v, (int, float)) and not isinstance(v, bool) and k.replace("_", "").isalnum():
                fields.setdefault(k, []).append(f'{prefix}_{k}{{stage="{name}"}} {v}')
    out = []
    for k, lines in fields.items():
        out.append(f"# TYPE {prefix}_{k} gauge")
        out += lines
    return "\n".join(out) + ("\n" if out else "")


def create_app(client: Client, model_name: str = "model") -> FastAPI:
    app = FastAPI(title="sglang-omni-b200")
    metrics = ServerMetrics()
    app.state.client = client
    app.state.metrics = metrics

    @app.get("/health")
    async def health():
        if not client.health():
            return JSONResponse({"status": "unhealthy"}, status_code=503)
        return {"status": "ok", **client.get_status()}

    @app.get("/metrics")
    async def get_metrics(format: str = "json"):
        """Request counters and latency percentiles of this server, and every stage's last load
        report (queue depth, requests in its engine, KV-cache pages in use)."""
        coord = getattr(client, "coordinator", None)
        stages = coord.latest_stage_stats() if coord is not None and hasattr(coord, "latest_stage_stats") else {}
        if format == "prometheus":
            return Response(content=metrics.prometheus() + stage_prometheus(stages),
                            media_type="text/plain; version=0.0.4")
        return {**metrics.snapshot(), "stages": stages}

    @app.get("/v1/models")
    async def models():
        return ModelList(data=[ModelCard(id=model_name, root=model_name)]).model_dump()

    @app.get("/playground")
    async def playground():
        """A single-page browser client of the chat endpoint (text / image / audio / video in,
        streamed text and speech out, the speech chunks played as they arrive)."""
        import pathlib

        html = (pathlib.Path(__file__).parent / "playground.html").read_text()
        return Response(content=html, media_type="text/html")

    @app.post("/v1/chat/completions")
    async def chat_completions(req: ChatCompletionRequest):
        greq = build_chat_generate_request(req)
        rid = greq.request_id or f"chatcmpl-{uuid.uuid4().hex[:20]}"
        greq.request_id = rid
        model = req.model or model_name
        if req.stream:
            return StreamingResponse(_chat_stream(client, greq, rid, model, metrics), media_type="text/event-stream")
        t0 = time.perf_counter()
        metrics.started()
        try:
            res = await client.completion(greq)
        except Exception as exc:
            metrics.failed()
            raise HTTPException(status_code=500, detail=str(exc)) from exc
        metrics.finished(time.perf_counter() - t0, None, res.usage.completion_tokens if res.usage else 0)
        msg: dict[str, Any] = {"role": "assistant", "content": res.text}
        if res.audio is not None:
            msg["audio"] = ChatCompletionAudio(id=res.audio.id, data=res.audio.data, transcript=res.text).model_dump()
        usage = UsageResponse(**(res.usage.to_dict() if res.usage else {}))
        return ChatCompletionResponse(id=rid, model=model, choices=[
            ChatCompletionChoice(message=msg, finish_reason=res.finish_reason)], usage=usage).model_dump(
            exclude_none=True)

    @app.post("/v1/audio/speech")
    async def create_speech(req: CreateSpeechRequest):
        greq = build_speech_generate_request(req)
        greq.request_id = f"speech-{uuid.uuid4().hex[:20]}"
        if req.stream:
            return StreamingResponse(_speech_stream(client, greq, req.response_format, metrics),
                                     media_type="text/event-stream")
        t0 = time.perf_counter()
        metrics.started()
        try:
            res = await client.speech(greq, req.response_format)
        except Exception as exc:
            metrics.failed()
            raise HTTPException(status_code=500, detail=str(exc)) from exc
        metrics.finished(time.perf_counter() - t0, None, res.usage.completion_tokens if res.usage else 0)
        headers = {}
        if res.usage is not None:
            headers = {"X-Prompt-Tokens": str(res.usage.prompt_tokens or 0),
                       "X-Completion-Tokens": str(res.usage.completion_tokens or 0),
                       "X-Engine-Time": f"{res.usage.engine_time_s or 0.0:.4f}"}
        return Response(content=res.audio_bytes, media_type=res.mime_type, headers=headers)

    return app


async def _chat_stream(client: Client, greq: GenerateRequest, rid: str, model: str, metrics: ServerMetrics):
    t0 = time.perf_counter()
    first_audio = first_text = last_text = None
    gaps: list[float] = []
    n_tokens = 0
    metrics.started()
    yield _sse(ChatCompletionStreamResponse(id=rid, model=model, choices=[
        ChatCompletionStreamChoice(delta=ChatCompletionStreamDelta(role="assistant", content=""))]))
    try:
        async for ch in client.completion_stream(greq):
            if ch.finish_reason is not None:
                usage = UsageResponse(**(ch.usage.to_dict() if ch.usage else {}))
                yield _sse(ChatCompletionStreamResponse(id=rid, model=model, choices=[
                    ChatCompletionStreamChoice(delta=ChatCompletionStreamDelta(), finish_reason=ch.finish_reason)],
                    usage=usage))
                n_tokens = usage.completion_tokens
                continue
            if ch.modality == "audio":
                if first_audio is None:
                    first_audio = time.perf_counter() - t0
                delta = ChatCompletionStreamDelta(audio=ChatCompletionAudio(id=f"audio-{rid}", data=ch.audio_b64))
            else:
                now = time.perf_counter()
                if first_text is None:
                    first_text = now - t0
                elif last_text is not None:
                    gaps.append(now - last_text)
                last_text = now
                delta = ChatCompletionStreamDelta(content=ch.text)
            yield _sse(ChatCompletionStreamResponse(id=rid, model=model,
                                                    choices=[ChatCompletionStreamChoice(delta=delta)]))
    except Exception as exc:
        metrics.failed()
        yield _sse({"error": {"message": str(exc), "type": "server_error"}})
    else:
        metrics.finished(time.perf_counter() - t0, first_audio, n_tokens, ttft_s=first_text,
                         itl_s=sum(gaps) / len(gaps) if gaps else None)
    yield "data: [DONE]\n\n"


async def _speech_stream(client: Client, greq: GenerateRequest, fmt: str, metrics: ServerMetrics):
    """SSE of ``/v1/audio/speech``: one ``audio.speech.chunk`` object per audio delta (its
    ``audio`` holds base64 data, format, mime type and sample rate), then a closing object
    with ``audio: null``, the finish reason and usage, then ``[DONE]``.  The terminal result
    carries the whole waveform: only its samples past those already streamed are sent."""
    t0 = time.perf_counter()
    first = None
    idx = 0
    sent = 0          # samples streamed so far
    finish, usage = None, None
    kind = "pcm" if fmt == "pcm" else "wav"
    sid = greq.request_id or f"speech-{uuid.uuid4().hex[:20]}"
    metrics.started()
    async for ch in client.generate(greq):
        terminal = ch.finish_reason is not None
        if terminal:
            finish = ch.finish_reason
            usage = ch.usage.to_dict() if ch.usage else None
        if ch.audio_data is not None:
            data = ch.audio_data
            if isinstance(data, (bytes, bytearray)):
                data = np.frombuffer(data, dtype=np.float32)
            data = np.asarray(data, dtype=np.float32).reshape(-1)
            if terminal:
                data = data[sent:]
            if data.size:
                if first is None:
                    first = time.perf_counter() - t0
                sent += data.size
                rate = ch.sample_rate or 24000
                audio = encode_audio(data, rate, kind)
                yield _sse({"id": sid, "object": "audio.speech.chunk", "index": idx,
                            "audio": {"data": base64.b64encode(audio).decode(), "format": kind,
                                      "mime_type": f"audio/{kind}", "sample_rate": rate},
                            "finish_reason": None})
                idx += 1
        if terminal:
            break
    metrics.finished(time.perf_counter() - t0, first, 0)
    yield _sse({"id": sid, "object": "audio.speech.chunk", "index": idx, "audio": None,
                "finish_reason": finish or "stop", "usage": usage})
    yield "data: [DONE]\n\n"
