"""Word / character error rate of synthesised speech: transcribe each clip with an ASR
model, normalise both texts, align them.

Normalisation: English uses transformers' Whisper ``EnglishTextNormalizer`` when it imports
(spelling map left empty: the map file is not shipped with transformers), else lowercasing,
punctuation removal and whitespace folding; Chinese compares characters without punctuation
or spaces (a character error rate).  The corpus rate pools edits over all samples; the
reference's report adds per-sample statistics and the share of samples above 50 % WER
(benchmarks/tasks/voice_clone.py:559-610), which ``wer_summary`` gives too.

ASR backends (no network here, so models load from a local directory only):
``whisper:<dir>`` (a Hugging Face Whisper checkpoint) or ``module:function`` (any callable
taking (float32 waveform, sample rate, language) and returning text)."""
from __future__ import annotations

import importlib
import re
import unicodedata
from dataclasses import dataclass
from typing import Callable

import numpy as np

_PUNCT = re.compile(r"[^\w\s']|_", re.UNICODE)


def _basic_en(text: str) -> str:
    text = unicodedata.normalize("NFKC", text).lower()
    text = _PUNCT.sub(" ", text).replace("'", "")
    return " ".join(text.split())


_EN: Callable[[str], str] | None = None


def normalize(text: str, lang: str = "en") -> str:
    global _EN
    if lang == "zh":
        text = unicodedata.normalize("NFKC", text)
        return "".join(ch for ch in text if not ch.isspace() and not unicodedata.category(ch).startswith("P"))
    if _EN is None:
        try:
            from transformers.models.whisper.english_normalizer import EnglishTextNormalizer

            _EN = EnglishTextNormalizer({})
        except Exception:
            _EN = _basic_en
    return " ".join(_EN(text).split())


@dataclass
class Alignment:
    hits: int
    substitutions: int
    deletions: int
    insertions: int

    @property
    def ref_len(self) -> int:
        return self.hits + self.substitutions + self.deletions

    @property
    def errors(self) -> int:
        return self.substitutions + self.deletions + self.insertions

    @property
    def rate(self) -> float:
        return self.errors / self.ref_len if self.ref_len else float(self.insertions > 0)


def align(ref: list[str], hyp: list[str]) -> Alignment:
    """Minimum-edit alignment (unit costs) with the edit kinds counted along one optimal path."""
    n, m = len(ref), len(hyp)
    d = np.zeros((n + 1, m + 1), dtype=np.int32)
    d[:, 0] = np.arange(n + 1)
    d[0, :] = np.arange(m + 1)
    for i in range(1, n + 1):
        for j in range(1, m + 1):
            d[i, j] = min(d[i - 1, j - 1] + (ref[i - 1] != hyp[j - 1]), d[i - 1, j] + 1, d[i, j - 1] + 1)
    i, j = n, m
    hit = sub = dele = ins = 0
    while i > 0 or j > 0:
        if i > 0 and j > 0 and d[i, j] == d[i - 1, j - 1] + (ref[i - 1] != hyp[j - 1]):
            if ref[i - 1] == hyp[j - 1]:
                hit += 1
            else:
                sub += 1
            i, j = i - 1, j - 1
        elif i > 0 and d[i, j] == d[i - 1, j] + 1:
            dele += 1
            i -= 1
        else:
            ins += 1
            j -= 1
    return Alignment(hit, sub, dele, ins)


def score(reference: str, hypothesis: str, lang: str = "en") -> Alignment:
    r, h = normalize(reference, lang), normalize(hypothesis, lang)
    if lang == "zh":
        return align(list(r), list(h))
    return align(r.split(), h.split())


def wer_summary(alignments: list[Alignment | None], lang: str = "en") -> dict:
    """Corpus and per-sample error rates (None entries are samples that produced no audio)."""
    ok = [a for a in alignments if a is not None]
    out = {"lang": lang, "total_samples": len(alignments), "evaluated": len(ok),
           "skipped": len(alignments) - len(ok)}
    if not ok:
        return out
    rates = np.array([a.rate for a in ok])
    ref = sum(a.ref_len for a in ok)
    out["wer_corpus"] = sum(a.errors for a in ok) / ref if ref else 0.0
    out["wer_per_sample_mean"] = float(rates.mean())
    out["wer_per_sample_median"] = float(np.median(rates))
    out["wer_per_sample_std"] = float(rates.std())
    out["wer_per_sample_p95"] = float(np.percentile(rates, 95))
    low = [a for a in ok if a.rate <= 0.5]
    low_ref = sum(a.ref_len for a in low)
    out["wer_below_50_corpus"] = sum(a.errors for a in low) / low_ref if low_ref else 0.0
    out["n_above_50_pct_wer"] = int((rates > 0.5).sum())
    out["pct_above_50_pct_wer"] = 100.0 * out["n_above_50_pct_wer"] / len(ok)
    return out


def load_asr(spec: str, device: str = "cpu") -> Callable[[np.ndarray, int, str], str]:
    """``whisper:<dir>`` or ``module:function`` (see the module docstring)."""
    kind, _, arg = spec.partition(":")
    if kind == "whisper":
        import torch
        from transformers import WhisperForConditionalGeneration, WhisperProcessor

        proc = WhisperProcessor.from_pretrained(arg, local_files_only=True)
        model = WhisperForConditionalGeneration.from_pretrained(arg, local_files_only=True).to(device).eval()

        def whisper(wave: np.ndarray, rate: int, lang: str) -> str:
            if rate != 16000:
                from ..preprocessing.media import resample

                wave = resample(wave, rate, 16000)
            feats = proc(wave, sampling_rate=16000, return_tensors="pt").input_features.to(device, model.dtype)
            with torch.no_grad():
                ids = model.generate(feats, language="zh" if lang == "zh" else "en", task="transcribe")
            return proc.batch_decode(ids, skip_special_tokens=True)[0]

        return whisper
    fn = getattr(importlib.import_module(kind), arg)
    return fn
