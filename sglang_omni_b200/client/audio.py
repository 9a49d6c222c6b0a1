"""Audio encoding for API responses: wav (16-bit PCM) and raw pcm natively,
other formats fall back to wav with the fallback reported
(sglang_omni/client/audio.py:132-226)."""
from __future__ import annotations

import base64
import io
import wave

import numpy as np

MIME = {"wav": "audio/wav", "pcm": "audio/pcm", "mp3": "audio/mpeg", "flac": "audio/flac", "opus": "audio/ogg",
        "aac": "audio/aac"}


def to_pcm16(wave_f32: np.ndarray) -> bytes:
    x = np.clip(np.asarray(wave_f32, dtype=np.float32).reshape(-1), -1.0, 1.0)
    return (x * 32767.0).astype("<i2").tobytes()


def encode_audio(wave_f32, sample_rate: int, fmt: str = "wav", return_meta: bool = False):
    fmt = (fmt or "wav").lower()
    if fmt == "pcm":
        data, used = to_pcm16(wave_f32), "pcm"
    else:
        buf = io.BytesIO()
        with wave.open(buf, "wb") as w:
            w.setnchannels(1)
            w.setsampwidth(2)
            w.setframerate(int(sample_rate))
            w.writeframes(to_pcm16(wave_f32))
        data, used = buf.getvalue(), "wav"
    if return_meta:
        return data, used, MIME[used]
    return data


def audio_to_base64(wave_f32, sample_rate: int, fmt: str = "wav") -> str:
    return base64.b64encode(encode_audio(wave_f32, sample_rate, fmt)).decode()


def decode_wav(data: bytes) -> tuple[np.ndarray, int]:
    with wave.open(io.BytesIO(data), "rb") as w:
        sr = w.getframerate()
        n = w.getnframes()
        width = w.getsampwidth()
        raw = w.readframes(n)
        ch = w.getnchannels()
    if width == 2:
        x = np.frombuffer(raw, dtype="<i2").astype(np.float32) / 32768.0
    elif width == 4:
        x = np.frombuffer(raw, dtype="<i4").astype(np.float32) / 2147483648.0
    else:
        x = (np.frombuffer(raw, dtype=np.uint8).astype(np.float32) - 128.0) / 128.0
    if ch > 1:
        x = x.reshape(-1, ch).mean(1)
    return x, sr
