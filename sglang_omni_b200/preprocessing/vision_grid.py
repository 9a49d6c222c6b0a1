"""Target sizes of images and video frames before patching, as the checkpoint's Hugging Face
image / video processors choose them (so the number of vision tokens, and every position after
them, matches what the model was trained with).

Rule (Qwen2-VL family processors): round each side to a multiple of ``factor`` (patch x merge);
if the area exceeds ``max_pixels`` scale both sides down by sqrt(area / max_pixels) and floor to
the factor, if it is below ``min_pixels`` scale up by sqrt(min_pixels / area) and ceil to the
factor.  The bounds come from the checkpoint's ``preprocessor_config.json`` (images) and
``video_preprocessor_config.json`` (videos), as ``min_pixels`` / ``max_pixels`` or
``size.shortest_edge`` / ``size.longest_edge``; without them the Qwen3-Omni processor defaults
apply (images 56^2 .. 3584^2 pixels, video frames 128 .. 768 blocks of 32 x 32)."""
from __future__ import annotations

import functools
import json
import math
import os
from dataclasses import dataclass

IMAGE_MIN_PIXELS = 56 * 56
IMAGE_MAX_PIXELS = 12845056
VIDEO_MIN_PIXELS = 128 * 32 * 32
VIDEO_MAX_PIXELS = 768 * 32 * 32


def resize_grid(height: int, width: int, factor: int, min_pixels: int = IMAGE_MIN_PIXELS,
                max_pixels: int = IMAGE_MAX_PIXELS) -> tuple[int, int]:
    """(target height, target width), both multiples of ``factor``."""
    if min(height, width) <= 0:
        raise ValueError(f"empty image {height}x{width}")
    if max(height, width) > 200 * min(height, width):
        raise ValueError(f"aspect ratio of a {height}x{width} image exceeds 200")
    th, tw = round(height / factor) * factor, round(width / factor) * factor
    if th * tw > max_pixels:
        s = math.sqrt(height * width / max_pixels)
        th, tw = math.floor(height / s / factor) * factor, math.floor(width / s / factor) * factor
    elif th * tw < min_pixels:
        s = math.sqrt(min_pixels / (height * width))
        th, tw = math.ceil(height * s / factor) * factor, math.ceil(width * s / factor) * factor
    return max(factor, th), max(factor, tw)


@dataclass(frozen=True)
class ResizeBounds:
    image_min: int = IMAGE_MIN_PIXELS
    image_max: int = IMAGE_MAX_PIXELS
    video_min: int = VIDEO_MIN_PIXELS
    video_max: int = VIDEO_MAX_PIXELS


def _bounds(d: dict, lo: int, hi: int) -> tuple[int, int]:
    size = d.get("size") or {}
    lo = d.get("min_pixels") or size.get("shortest_edge") or lo
    hi = d.get("max_pixels") or size.get("longest_edge") or hi
    return int(lo), int(hi)


@functools.lru_cache(maxsize=16)
def checkpoint_bounds(model_path: str | None) -> ResizeBounds:
    """Bounds of a checkpoint directory (defaults for anything else, e.g. random weights)."""
    b = ResizeBounds()
    if not model_path or not os.path.isdir(model_path):
        return b
    img, vid = (b.image_min, b.image_max), (b.video_min, b.video_max)
    p = os.path.join(model_path, "preprocessor_config.json")
    if os.path.exists(p):
        with open(p) as f:
            img = _bounds(json.load(f), *img)
    p = os.path.join(model_path, "video_preprocessor_config.json")
    if os.path.exists(p):
        with open(p) as f:
            vid = _bounds(json.load(f), *vid)
    return ResizeBounds(img[0], img[1], vid[0], vid[1])
