"""Benchmark inputs: seed-tts-eval ``meta.lst`` files and synthetic sentences.

``meta.lst`` holds one sample per line, ``id|reference text|reference wav (relative to the
file)|target text`` (the format the reference reads in benchmarks/dataset/seedtts.py)."""
from __future__ import annotations

import os
import random
from dataclasses import dataclass


@dataclass
class SpeechSample:
    sample_id: str
    target_text: str
    ref_text: str = ""
    ref_audio: str = ""        # path or URL of the voice-cloning reference ("" = none)


def load_meta_lst(path: str, limit: int | None = None) -> list[SpeechSample]:
    root = os.path.dirname(os.path.abspath(path))
    out: list[SpeechSample] = []
    with open(path, encoding="utf-8") as f:
        for raw in f:
            fields = raw.rstrip("\n").split("|")
            if len(fields) < 4 or not fields[0].strip():
                continue
            sid, ref_text, wav, target = (x.strip() for x in fields[:4])
            ref = wav if (not wav or "://" in wav or os.path.isabs(wav)) else os.path.join(root, wav)
            out.append(SpeechSample(sid, target, ref_text, ref))
            if limit is not None and len(out) >= limit:
                break
    return out


_WORDS = ("the quick brown fox jumps over a lazy dog while seven bright lanterns glow along the quiet "
          "harbour and distant bells ring through the cold morning air as travellers gather near the "
          "old stone bridge to watch ships return from the northern sea").split()


def synthetic_samples(n: int, words: int = 24, seed: int = 0) -> list[SpeechSample]:
    """``n`` English sentences of ``words`` words (no dataset download needed)."""
    rnd = random.Random(seed)
    return [SpeechSample(f"synthetic-{i}", " ".join(rnd.choice(_WORDS) for _ in range(words)).capitalize() + ".")
            for i in range(n)]
