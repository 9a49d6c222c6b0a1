"""Cache keys of request media, so an encoder stage can reuse the output of media it has
already encoded (its engine keeps an LRU of outputs by key).

A key covers every item of one modality of a request, in order, plus the preprocessing
context that changes the encoder input (sample rate, patch / merge unit, video frame rate...):
the same clip under other settings is another key.  Items are fingerprinted by content:

* arrays / tensors / PIL images / raw bytes: dtype, shape and a BLAKE2b digest of every byte;
* local files: size and a digest of the whole file (files over 256 MiB: the first and last
  16 MiB and the size);
* URLs: the URL text (their content is fetched through the media LRU, which keys by URL too);
* data URIs and base64 strings: the text.

An item of another type gives no key (the request is encoded, not cached).  The reference
keys media the same way in spirit (sglang_omni/preprocessing/cache_key.py:27-112: xxhash of
sampled files and array contents); the digests here are BLAKE2b from hashlib."""
from __future__ import annotations

import hashlib
import os
from typing import Any

import numpy as np

_FULL_FILE = 256 << 20
_EDGE = 16 << 20


def _digest(*parts: bytes) -> str:
    h = hashlib.blake2b(digest_size=16)
    for p in parts:
        h.update(p)
    return h.hexdigest()


def _file(path: str) -> str:
    size = os.path.getsize(path)
    h = hashlib.blake2b(digest_size=16)
    h.update(str(size).encode())
    with open(path, "rb") as f:
        if size <= _FULL_FILE:
            for block in iter(lambda: f.read(1 << 20), b""):
                h.update(block)
        else:
            h.update(f.read(_EDGE))
            f.seek(size - _EDGE)
            h.update(f.read(_EDGE))
    return "file:" + h.hexdigest()


def fingerprint(item: Any) -> str | None:
    """Content fingerprint of one media item, or None when it cannot be keyed."""
    if isinstance(item, (bytes, bytearray, memoryview)):
        return "bytes:" + _digest(bytes(item))
    if isinstance(item, str):
        if item.startswith(("http://", "https://")):
            return "url:" + _digest(item.encode())
        path = item[7:] if item.startswith("file://") else item
        if not item.startswith("data:") and len(path) < 4096 and os.path.isfile(path):
            return _file(path)
        return "text:" + _digest(item.encode())
    if isinstance(item, np.ndarray):
        a = np.ascontiguousarray(item)
        return f"np:{a.dtype}:{a.shape}:" + _digest(a.view(np.uint8).reshape(-1).data if a.size else b"")
    try:
        import torch

        if isinstance(item, torch.Tensor):
            t = item.detach().contiguous().cpu()
            raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
            return f"pt:{t.dtype}:{tuple(t.shape)}:" + _digest(raw)
    except ImportError:
        pass
    try:
        from PIL import Image

        if isinstance(item, Image.Image):
            return f"pil:{item.mode}:{item.size}:" + _digest(item.tobytes())
    except ImportError:
        pass
    if isinstance(item, dict):
        parts = []
        for k in sorted(item):
            f = fingerprint(item[k]) if not isinstance(item[k], (int, float, bool, type(None))) else repr(item[k])
            if f is None:
                return None
            parts.append(f"{k}={f}")
        return "dict:" + _digest("|".join(parts).encode())
    return None


def media_cache_key(kind: str, items: list, **context: Any) -> str | None:
    """Key of all ``items`` of one modality under ``context``; None if there are no items or
    one of them cannot be fingerprinted."""
    if not items:
        return None
    prints = []
    for it in items:
        f = fingerprint(it)
        if f is None:
            return None
        prints.append(f)
    ctx = ",".join(f"{k}={context[k]!r}" for k in sorted(context))
    return f"{kind}:" + _digest(ctx.encode(), b"|", "|".join(prints).encode())
