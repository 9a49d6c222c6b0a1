"""Media inputs of the preprocessing stages: resource fetching, video decoding
and frame sampling, audio decoding and resampling.

* ``fetch(src)``: bytes of an ``http(s)://`` URL (bounded timeout and size), a
  ``file://`` URL or path, or a ``data:`` URI; results of URL fetches are kept
  in a small LRU keyed by the URL (the reference's resource connector and
  cache keys: sglang_omni/preprocessing/resource_connector.py:64,
  preprocessing/cache_key.py:27).
* ``load_video(item)``: uint8 RGB frames [N, H, W, 3] sampled at ``fps``
  (default 2, the Qwen3-Omni processor's rate), N rounded up to a multiple of
  the temporal patch (2) by repeating the last frame, plus the seconds covered
  by one temporal patch (``second_per_grid``).  Items: a frame array, a dict
  ``{"frames": ..., "fps": ...}``, or an encoded file (path / URL / bytes)
  decoded with OpenCV (sglang_omni/preprocessing/video.py:101).
* ``load_audio(item)``: float32 mono at 16 kHz from an array, a dict
  ``{"array", "sampling_rate"}`` or WAV bytes / path / URL; other rates are
  resampled with a polyphase filter (sglang_omni/preprocessing/audio.py:147-261).
  Only WAV is decoded: this build has no compressed-audio codec library.
"""
from __future__ import annotations

import base64
import os
import tempfile
import threading
import urllib.request
from collections import OrderedDict
from fractions import Fraction
from typing import Any

import numpy as np

SAMPLE_RATE = 16000
VIDEO_FPS = 2.0
TEMPORAL_PATCH = 2
MAX_FETCH_BYTES = 512 << 20
FETCH_TIMEOUT_S = 30.0

_cache_lock = threading.Lock()
_cache: "OrderedDict[str, bytes]" = OrderedDict()
_CACHE_BYTES = 256 << 20


def _cache_get(key: str) -> bytes | None:
    with _cache_lock:
        v = _cache.get(key)
        if v is not None:
            _cache.move_to_end(key)
        return v


def _cache_put(key: str, data: bytes) -> None:
    with _cache_lock:
        _cache[key] = data
        total = sum(len(v) for v in _cache.values())
        while total > _CACHE_BYTES and len(_cache) > 1:
            _, old = _cache.popitem(last=False)
            total -= len(old)


def is_url(s: str) -> bool:
    return s.startswith(("http://", "https://", "file://", "data:"))


def fetch(src: str, timeout_s: float = FETCH_TIMEOUT_S) -> bytes:
    """Bytes of a URL / data URI / local path."""
    if src.startswith("data:"):
        return base64.b64decode(src.split(",", 1)[1])
    if src.startswith("file://"):
        src = src[len("file://"):]
    if not src.startswith(("http://", "https://")):
        with open(src, "rb") as f:
            return f.read()
    hit = _cache_get(src)
    if hit is not None:
        return hit
    with urllib.request.urlopen(src, timeout=timeout_s) as r:
        data = r.read(MAX_FETCH_BYTES + 1)
    if len(data) > MAX_FETCH_BYTES:
        raise ValueError(f"{src}: resource larger than {MAX_FETCH_BYTES} bytes")
    _cache_put(src, data)
    return data


def _bytes_of(item: str) -> bytes:
    if is_url(item) or os.path.exists(item):
        return fetch(item)
    return base64.b64decode(item, validate=True)   # bare base64


# ----------------------------------------------------------------------------- video
def _decode_video(data: bytes) -> tuple[np.ndarray, float]:
    import cv2

    with tempfile.NamedTemporaryFile(suffix=".video", delete=False) as f:
        f.write(data)
        path = f.name
    try:
        cap = cv2.VideoCapture(path)
        if not cap.isOpened():
            raise ValueError("could not decode the video")
        fps = float(cap.get(cv2.CAP_PROP_FPS) or 0.0) or 25.0
        frames = []
        while True:
            ok, fr = cap.read()
            if not ok:
                break
            frames.append(fr[..., ::-1])       # BGR -> RGB
        cap.release()
    finally:
        os.unlink(path)
    if not frames:
        raise ValueError("the video has no frames")
    return np.ascontiguousarray(np.stack(frames)), fps


def sample_frames(frames: np.ndarray, src_fps: float, fps: float = VIDEO_FPS, max_frames: int = 768,
                  min_frames: int = 4) -> np.ndarray:
    """Frames at `fps` (nearest source frame), between min_frames and max_frames, count a
    multiple of the temporal patch (the last frame repeated)."""
    n = frames.shape[0]
    duration = n / max(src_fps, 1e-6)
    want = int(round(duration * fps))
    want = max(min(want, max_frames, n), min(min_frames, n), 1)
    idx = np.linspace(0, n - 1, want).round().astype(np.int64)
    out = frames[idx]
    pad = (-out.shape[0]) % TEMPORAL_PATCH
    if pad:
        out = np.concatenate([out, np.repeat(out[-1:], pad, 0)], 0)
    return out


def load_video(item: Any, fps: float = VIDEO_FPS, max_frames: int = 768) -> dict:
    """{"frames": uint8 [N, H, W, 3] (N a multiple of 2), "fps": sampled rate,
    "second_per_grid": seconds spanned by one temporal patch}."""
    src_fps = None
    if isinstance(item, dict):
        src_fps = item.get("fps")
        item = item.get("frames", item.get("url", item.get("video", item.get("data"))))
    if isinstance(item, (bytes, bytearray)):
        frames, src_fps = _decode_video(bytes(item))
    elif isinstance(item, str):
        frames, src_fps = _decode_video(_bytes_of(item))
    else:
        frames = np.asarray(item)
        if frames.dtype != np.uint8:
            frames = np.clip(frames, 0, 255).astype(np.uint8)
        if frames.ndim != 4 or frames.shape[-1] != 3:
            raise ValueError(f"video frames must be [N, H, W, 3], got {frames.shape}")
        src_fps = float(src_fps or fps)
    frames = sample_frames(frames, float(src_fps), fps, max_frames)
    return {"frames": frames, "fps": float(fps), "second_per_grid": TEMPORAL_PATCH / float(fps)}


# ----------------------------------------------------------------------------- audio
def resample(x: np.ndarray, sr: int, target: int = SAMPLE_RATE) -> np.ndarray:
    """Polyphase resampling (scipy.signal.resample_poly) to `target` Hz."""
    if sr == target:
        return x
    from scipy.signal import resample_poly

    fr = Fraction(target, sr).limit_denominator(1000)
    return resample_poly(x, fr.numerator, fr.denominator).astype(np.float32)


def _decode_audio(data: bytes) -> tuple[np.ndarray, int]:
    if data[:4] != b"RIFF":
        raise ValueError("only WAV audio can be decoded (no compressed-audio codec library in this build)")
    from ..client.audio import decode_wav

    try:
        return decode_wav(data)
    except Exception:
        import io

        from scipy.io import wavfile

        sr, x = wavfile.read(io.BytesIO(data))
        x = np.asarray(x)
        if x.dtype.kind in "iu":
            x = x.astype(np.float32) / float(np.iinfo(x.dtype).max)
        x = x.astype(np.float32)
        if x.ndim == 2:
            x = x.mean(1)
        return x, int(sr)


def load_audio(item: Any, target_sr: int = SAMPLE_RATE) -> np.ndarray:
    sr = target_sr
    if isinstance(item, dict):
        sr = int(item.get("sampling_rate", target_sr))
        item = item.get("array", item.get("data", item.get("url", item.get("path"))))
    if isinstance(item, (bytes, bytearray)):
        x, sr = _decode_audio(bytes(item))
    elif isinstance(item, str):
        x, sr = _decode_audio(_bytes_of(item))
    else:
        x = np.asarray(item, dtype=np.float32).reshape(-1)
    x = np.asarray(x, dtype=np.float32).reshape(-1)
    return resample(x, int(sr), target_sr)


def video_grid(frames: np.ndarray, unit: int, max_pixels: int | None = None,
               min_pixels: int | None = None) -> tuple[int, int, int]:
    """Merged (t, h, w) token grid of sampled frames: each frame resized to the video
    processor's target size (a multiple of `unit` = patch x merge within the pixel bounds,
    ``vision_grid.resize_grid``)."""
    from .vision_grid import VIDEO_MAX_PIXELS, VIDEO_MIN_PIXELS, resize_grid

    n, H, W = frames.shape[:3]
    th, tw = resize_grid(H, W, unit, VIDEO_MIN_PIXELS if min_pixels is None else min_pixels,
                         VIDEO_MAX_PIXELS if max_pixels is None else max_pixels)
    return n // TEMPORAL_PATCH, th // unit, tw // unit
