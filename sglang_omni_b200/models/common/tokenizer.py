"""Tokenizer adapters (sglang_omni/engines/omni/runtime/tokenizer.py:20-116).

``load_tokenizer(model_path)`` returns the HF tokenizer of a checkpoint when
its files are present, else a deterministic byte-level fallback so random-init
deployments (benchmarks, tests) serve text end to end.
"""
from __future__ import annotations

import os


class ByteTokenizer:
    """UTF-8 bytes shifted into [offset, offset + 256); ids outside decode as <id>."""

    def __init__(self, vocab_size: int = 151936, offset: int = 3, eos_token_id: int = 2):
        self.vocab_size = vocab_size
        self.offset = offset
        self.eos_token_id = eos_token_id

    def encode(self, text: str) -> list[int]:
        return [b + self.offset for b in text.encode("utf-8")]

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        out = bytearray()
        parts = []
        for i in ids:
            i = int(i)
            if self.offset <= i < self.offset + 256:
                out.append(i - self.offset)
            else:
                if out:
                    parts.append(out.decode("utf-8", errors="replace"))
                    out = bytearray()
                parts.append(f"<{i}>")
        if out:
            parts.append(out.decode("utf-8", errors="replace"))
        return "".join(parts)

    def apply_chat_template(self, messages, add_generation_prompt=True, tokenize=False, **_):
        text = ""
        for m in messages:
            content = m["content"] if isinstance(m, dict) else m.content
            if isinstance(content, list):
                content = "".join(c.get("text", "") for c in content if isinstance(c, dict))
            role = m["role"] if isinstance(m, dict) else m.role
            text += f"<|im_start|>{role}\n{content}<|im_end|>\n"
        if add_generation_prompt:
            text += "<|im_start|>assistant\n"
        return self.encode(text) if tokenize else text


def load_tokenizer(model_path: str | None, vocab_size: int = 151936):
    if model_path and os.path.isdir(model_path) and any(
            os.path.exists(os.path.join(model_path, f)) for f in ("tokenizer.json", "tokenizer_config.json")):
        from transformers import AutoTokenizer

        return AutoTokenizer.from_pretrained(model_path, trust_remote_code=False)
    return ByteTokenizer(vocab_size)


class IncrementalDetokenizer:
    """Emits only complete UTF-8 text (holds back a trailing replacement char),
    like decode_events in sglang_omni/models/qwen3_omni/pipeline/merge.py:248."""

    def __init__(self, tokenizer):
        self.tok = tokenizer
        self.ids: list[int] = []
        self.emitted = 0

    def push(self, token_id: int) -> str:
        self.ids.append(int(token_id))
        text = self.tok.decode(self.ids, skip_special_tokens=True)
        if text.endswith("�"):
            return ""
        delta = text[self.emitted:]
        self.emitted = len(text)
        return delta


class SpecialsByteTokenizer(ByteTokenizer):
    """ByteTokenizer that also maps a fixed list of special-token strings to ids
    ``base, base + 1, ...`` (for random-init deployments of models whose prompts
    are built from special tokens)."""

    def __init__(self, specials: list[str], vocab_size: int, base: int | None = None, eos: str | None = None):
        super().__init__(vocab_size)
        import re

        base = base if base is not None else vocab_size - len(specials) - 1
        if base < self.offset + 256:
            raise ValueError("vocabulary too small for bytes and special tokens")
        self._tok2id = {s: base + i for i, s in enumerate(specials)}
        self._id2tok = {v: k for k, v in self._tok2id.items()}
        self._re = re.compile("(" + "|".join(re.escape(s) for s in sorted(specials, key=len, reverse=True)) + ")")
        if eos is not None:
            self.eos_token_id = self._tok2id[eos]

    def convert_tokens_to_ids(self, token):
        if isinstance(token, (list, tuple)):
            return [self.convert_tokens_to_ids(t) for t in token]
        return self._tok2id[token]

    def encode(self, text: str, add_special_tokens: bool = False) -> list[int]:
        ids: list[int] = []
        for piece in self._re.split(text):
            if not piece:
                continue
            if piece in self._tok2id:
                ids.append(self._tok2id[piece])
            else:
                ids.extend(super().encode(piece))
        return ids

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        out, run = [], []
        for i in ids:
            i = int(i)
            if i in self._id2tok:
                if run:
                    out.append(super().decode(run))
                    run = []
                if not skip_special_tokens:
                    out.append(self._id2tok[i])
            else:
                run.append(i)
        if run:
            out.append(super().decode(run))
        return "".join(out)
