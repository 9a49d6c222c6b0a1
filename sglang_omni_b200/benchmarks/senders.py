"""HTTP requests of the benchmark tasks and the parsing of their responses.

* ``speech``: ``POST /v1/audio/speech`` (S2-Pro-style TTS).  Non-streamed: a WAV body and the
  ``X-Prompt-Tokens`` / ``X-Completion-Tokens`` / ``X-Engine-Time`` headers.  Streamed: SSE
  ``audio.speech.chunk`` objects whose ``audio.data`` is a base64 WAV (or PCM) piece, and a
  closing object with usage.
* ``omni_chat``: ``POST /v1/chat/completions`` with ``modalities: ["text", "audio"]``
  (Qwen3-Omni speech out).  Non-streamed: ``message.audio.data`` (base64 WAV) and
  ``message.content``; streamed: ``delta.content`` / ``delta.audio.data`` chunks, usage last.
  Voice cloning sends the reference clip in ``audios`` with a read-aloud instruction, as the
  reference's VoiceCloneOmni does (benchmarks/tasks/voice_clone.py:431-513).
"""
from __future__ import annotations

import base64
import json
import os
import time

import numpy as np

from ..client.audio import decode_wav, encode_audio
from .datasets import SpeechSample
from .results import RequestOutcome


def wav_seconds(data: bytes) -> float:
    try:
        x, sr = decode_wav(data)
    except Exception:
        return 0.0
    return x.shape[0] / sr if sr else 0.0


def _pcm_seconds(data: bytes, rate: int) -> float:
    return len(data) / 2 / rate if rate else 0.0


async def _sse_events(resp):
    """JSON objects of an SSE body (``data: {...}`` lines; ``[DONE]`` ends it)."""
    buf = b""
    async for piece in resp.content.iter_any():
        buf += piece
        while b"\n" in buf:
            line, buf = buf.split(b"\n", 1)
            line = line.strip()
            if not line.startswith(b"data:"):
                continue
            body = line[5:].strip()
            if body == b"[DONE]":
                return
            if body:
                yield json.loads(body)
    tail = buf.strip()
    if tail.startswith(b"data:") and tail[5:].strip() not in (b"", b"[DONE]"):
        yield json.loads(tail[5:].strip())


def _usage_into(out: RequestOutcome, usage: dict | None) -> None:
    if not usage:
        return
    out.prompt_tokens = int(usage.get("prompt_tokens") or 0)
    out.completion_tokens = int(usage.get("completion_tokens") or 0)
    out.engine_time_s = float(usage.get("engine_time_s") or 0.0)


def _save(out: RequestOutcome, save_dir: str | None, pieces: list[np.ndarray], rate: int) -> None:
    if save_dir and pieces:
        os.makedirs(save_dir, exist_ok=True)
        path = os.path.join(save_dir, f"{out.request_id}.wav")
        with open(path, "wb") as f:
            f.write(encode_audio(np.concatenate(pieces), rate, "wav"))
        out.wav_path = path


def _piece(data: bytes, fmt: str, rate: int) -> tuple[np.ndarray, int]:
    if fmt == "pcm":
        return np.frombuffer(data, dtype="<i2").astype(np.float32) / 32768.0, rate
    return decode_wav(data)


async def speech(session, base_url: str, sample: SpeechSample, request_id: str, *, model: str = "default",
                 stream: bool = False, params: dict | None = None, use_reference: bool = True,
                 save_dir: str | None = None) -> RequestOutcome:
    body = {"model": model, "input": sample.target_text, "response_format": "wav"}
    if use_reference and sample.ref_audio:
        body["ref_audio"], body["ref_text"] = sample.ref_audio, sample.ref_text
    body.update({k: v for k, v in (params or {}).items() if v is not None})
    if stream:
        body["stream"] = True
    out = RequestOutcome(request_id=request_id, text=sample.target_text)
    t0 = time.perf_counter()
    async with session.post(f"{base_url}/v1/audio/speech", json=body) as resp:
        if resp.status != 200:
            out.error = f"HTTP {resp.status}: {(await resp.text())[:300]}"
            return out
        pieces, rate = [], 24000
        if not stream:
            data = await resp.read()
            out.latency_s = time.perf_counter() - t0
            h = resp.headers
            out.prompt_tokens = int(h.get("X-Prompt-Tokens") or 0)
            out.completion_tokens = int(h.get("X-Completion-Tokens") or 0)
            out.engine_time_s = float(h.get("X-Engine-Time") or 0.0)
            x, rate = _piece(data, "wav", 0)
            pieces.append(x)
            out.audio_s = x.shape[0] / rate if rate else 0.0
        else:
            async for ev in _sse_events(resp):
                audio = ev.get("audio")
                if isinstance(audio, dict) and audio.get("data"):
                    if out.ttfa_s is None:
                        out.ttfa_s = time.perf_counter() - t0
                    rate = int(audio.get("sample_rate") or rate)
                    x, r = _piece(base64.b64decode(audio["data"]), audio.get("format", "wav"), rate)
                    rate = r or rate
                    pieces.append(x)
                    out.audio_s += x.shape[0] / rate if rate else 0.0
                if ev.get("usage"):
                    _usage_into(out, ev["usage"])
            out.latency_s = time.perf_counter() - t0
    out.ok = out.audio_s > 0
    if not out.ok:
        out.error = "no audio in the response"
    _save(out, save_dir, pieces, rate)
    return out


def read_aloud_prompt(sample: SpeechSample, lang: str, clone: bool) -> str:
    if lang == "zh":
        if clone:
            return f"听上面的音频，说话人正在朗读：“{sample.ref_text}”。请用同样的声音朗读下面的文本：{sample.target_text}"
        return f"请用中文朗读下面的文本：{sample.target_text}"
    if clone:
        return (f'Listen to the audio above; the speaker reads: "{sample.ref_text}". Read the following text '
                f"aloud in the same voice and style: {sample.target_text}")
    return f"Read the following text aloud in English: {sample.target_text}"


async def omni_chat(session, base_url: str, sample: SpeechSample, request_id: str, *, model: str = "default",
                    stream: bool = False, lang: str = "en", max_tokens: int = 256, temperature: float = 0.7,
                    use_reference: bool = True, save_dir: str | None = None,
                    params: dict | None = None) -> RequestOutcome:
    clone = bool(use_reference and sample.ref_audio)
    body = {"model": model, "messages": [{"role": "user", "content": read_aloud_prompt(sample, lang, clone)}],
            "modalities": ["text", "audio"], "audio": {"format": "wav"}, "max_tokens": max_tokens,
            "temperature": temperature, "stream": stream}
    if clone:
        body["audios"] = [sample.ref_audio]
    body.update({k: v for k, v in (params or {}).items() if v is not None})
    out = RequestOutcome(request_id=request_id)
    pieces, rate, text = [], 24000, []
    t0 = time.perf_counter()
    async with session.post(f"{base_url}/v1/chat/completions", json=body) as resp:
        if resp.status != 200:
            out.error = f"HTTP {resp.status}: {(await resp.text())[:300]}"
            return out
        if not stream:
            js = await resp.json()
            out.latency_s = time.perf_counter() - t0
            msg = (js.get("choices") or [{}])[0].get("message") or {}
            text.append(msg.get("content") or "")
            audio = msg.get("audio") or {}
            if audio.get("data"):
                x, rate = decode_wav(base64.b64decode(audio["data"]))
                pieces.append(x)
            _usage_into(out, js.get("usage"))
        else:
            async for ev in _sse_events(resp):
                for ch in ev.get("choices") or []:
                    delta = ch.get("delta") or {}
                    if delta.get("content"):
                        if out.ttft_s is None:
                            out.ttft_s = time.perf_counter() - t0
                        text.append(delta["content"])
                    audio = delta.get("audio") or {}
                    if audio.get("data"):
                        if out.ttfa_s is None:
                            out.ttfa_s = time.perf_counter() - t0
                        x, rate = decode_wav(base64.b64decode(audio["data"]))
                        pieces.append(x)
                if ev.get("usage"):
                    _usage_into(out, ev["usage"])
            out.latency_s = time.perf_counter() - t0
    out.text = "".join(text)
    out.audio_s = sum(p.shape[0] for p in pieces) / rate if rate else 0.0
    out.ok = out.audio_s > 0
    if not out.ok:
        out.error = "no audio in the response"
    _save(out, save_dir, pieces, rate)
    return out
