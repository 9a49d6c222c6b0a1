"""Thinker request construction: prompt layout with audio / image placeholders
and 3-D M-RoPE positions.

Positions follow the Qwen3-Omni rules (transformers get_rope_index, used by
sglang_omni/models/qwen3_omni/pipeline/engine_io.py:94-151): text and audio
tokens advance all three rows together; an image contributes (t, h, w) grid
positions on its merged patch grid starting at the running index, and the
text after it restarts at max + 1.  Without images or videos the positions
are plain 0..L-1 and the decode delta is 0.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from .hf_config import (AUDIO_START_TOKEN_ID, AUDIO_TOKEN_ID, IMAGE_TOKEN_ID, VIDEO_TOKEN_ID,
                        VISION_START_TOKEN_ID)

AUDIO_END_TOKEN_ID = 151648
VISION_END_TOKEN_ID = 151653
IM_START, IM_END, NEWLINE = 151644, 151645, 198
SYSTEM_ID, USER_ID, ASSISTANT_ID = 8948, 872, 77091


@dataclass
class PromptLayout:
    ids: list[int]
    audio_spans: list[tuple[int, int]] = field(default_factory=list)   # [start, end) of audio pad tokens
    image_spans: list[tuple[int, int]] = field(default_factory=list)
    image_grids: list[tuple[int, int, int]] = field(default_factory=list)  # merged (t, h, w)
    video_spans: list[tuple[int, int]] = field(default_factory=list)
    video_grids: list[tuple[int, int, int]] = field(default_factory=list)  # merged (t, h, w)
    video_second_per_grid: list[float] = field(default_factory=list)       # seconds per temporal patch


def build_prompt(tokenizer, messages: list[dict] | None, text: str | None, audio_tokens: list[int],
                 image_grids: list[tuple[int, int, int]] | None = None, system: str | None = None,
                 video_grids: list[tuple[int, int, int]] | None = None,
                 video_second_per_grid: list[float] | None = None) -> PromptLayout:
    """Chat-template layout: [system] user (images, videos, audios, text) then the assistant header.

    Media placeholders are inserted before the text of the last user turn (as
    the reference preprocessor does, models/qwen3_omni/components/preprocessor.py:128)."""
    image_grids = image_grids or []
    video_grids = video_grids or []
    spg = list(video_second_per_grid or [1.0] * len(video_grids))
    enc = (lambda s: list(tokenizer.encode(s))) if tokenizer is not None else (lambda s: [])
    ids: list[int] = []
    lay = PromptLayout(ids)
    if system:
        ids += [IM_START, SYSTEM_ID, NEWLINE] + enc(system) + [IM_END, NEWLINE]
    turns = messages or [{"role": "user", "content": text or ""}]
    last_user = max((i for i, m in enumerate(turns) if m.get("role") == "user"), default=-1)
    for i, m in enumerate(turns):
        role = m.get("role", "user")
        rid = {"system": SYSTEM_ID, "user": USER_ID, "assistant": ASSISTANT_ID}.get(role, USER_ID)
        content = m.get("content") or ""
        if isinstance(content, list):
            content = "".join(c.get("text", "") for c in content if isinstance(c, dict) and c.get("type") == "text")
        ids += [IM_START, rid, NEWLINE]
        if i == last_user:
            for (t, h, w) in image_grids:
                n = t * h * w
                ids.append(VISION_START_TOKEN_ID)
                lay.image_spans.append((len(ids), len(ids) + n))
                lay.image_grids.append((t, h, w))
                ids += [IMAGE_TOKEN_ID] * n
                ids.append(VISION_END_TOKEN_ID)
            for (t, h, w), sec in zip(video_grids, spg):
                n = t * h * w
                ids.append(VISION_START_TOKEN_ID)
                lay.video_spans.append((len(ids), len(ids) + n))
                lay.video_grids.append((t, h, w))
                lay.video_second_per_grid.append(float(sec))
                ids += [VIDEO_TOKEN_ID] * n
                ids.append(VISION_END_TOKEN_ID)
            for n in audio_tokens:
                ids.append(AUDIO_START_TOKEN_ID)
                lay.audio_spans.append((len(ids), len(ids) + n))
                ids += [AUDIO_TOKEN_ID] * n
                ids.append(AUDIO_END_TOKEN_ID)
        ids += enc(content) + [IM_END, NEWLINE]
    ids += [IM_START, ASSISTANT_ID, NEWLINE]
    return lay


def mrope_positions(lay: PromptLayout, position_id_per_seconds: int = 25) -> tuple[torch.Tensor, int]:
    """[3, L] int32 positions and the decode delta (next position - L).

    A video's temporal rows advance by second_per_grid * position_id_per_seconds per
    temporal patch (an image's by position_id_per_seconds); the positions are rounded to
    integers (exact for the default 2 fps sampling: 25 per patch)."""
    L = len(lay.ids)
    if not lay.image_spans and not lay.video_spans:
        p = torch.arange(L, dtype=torch.int32)
        return torch.stack([p, p, p]), 0
    visual = [(a, b, g, float(position_id_per_seconds)) for (a, b), g in zip(lay.image_spans, lay.image_grids)]
    visual += [(a, b, g, sec * position_id_per_seconds)
               for (a, b), g, sec in zip(lay.video_spans, lay.video_grids, lay.video_second_per_grid)]
    visual.sort(key=lambda v: v[0])
    pos = np.zeros((3, L), dtype=np.int64)
    cur = 0
    st = 0
    for a, b, (t, h, w), t_step in visual:
        n = a - st
        pos[:, st:a] = np.arange(n)[None] + cur
        cur += n
        tt = np.repeat(np.rint(np.arange(t) * t_step).astype(np.int64), h * w)
        hh = np.tile(np.repeat(np.arange(h), w), t)
        ww = np.tile(np.arange(w), t * h)
        pos[0, a:b] = tt + cur
        pos[1, a:b] = hh + cur
        pos[2, a:b] = ww + cur
        cur = int(pos[:, a:b].max()) + 1
        st = b
    n = L - st
    pos[:, st:] = np.arange(n)[None] + cur
    delta = int(pos.max()) + 1 - L
    return torch.from_numpy(pos.astype(np.int32)), delta
