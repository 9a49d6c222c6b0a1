"""S2-Pro prompt construction (Qwen3 chat layout with VQ parts).

The prompt is a sequence of parts, each encoded on its own:

    [system, only with voice-cloning references]
      "<|im_start|>system\\n"
      "convert the provided text to speech reference to the following:\\n\\nText:\\n"
      "<|speaker:S|>{reference text}"          (one per reference with text)
      "\\n\\nSpeech:\\n"
      VQ part: one <|semantic:c0|> token per reference frame   (vq_mask = 1)
      "<|im_end|>\\n"
    "<|im_start|>user\\n" "<|speaker:S|>{text}" "<|im_end|>\\n"
    "<|im_start|>assistant\\n<|voice|>"          (generation starts here)

which is what S2ProTokenizerAdapter.build_prompt produces through the fish
Conversation / ContentSequence encoders (sglang_omni/models/fishaudio_s2_pro/
tokenizer.py:56-143, fish_speech/conversation.py:44-75,
fish_speech/content_sequence.py:192-300).  VQ positions carry all codebooks
of their frame (``vq_codes`` rows, [n_vq, num_codebooks]); the engine adds
their codebook embeddings to the token embedding.

With a checkpoint directory the HF tokenizer is used; otherwise a
deterministic fallback (UTF-8 bytes + the special tokens at fixed ids, the
semantic tokens contiguous from ``semantic_begin_id``) keeps random-init
deployments serving end to end.
"""
from __future__ import annotations

import os
import re
from dataclasses import dataclass

import torch

IM_START = "<|im_start|>"
IM_END = "<|im_end|>"
VOICE = "<|voice|>"
SEMANTIC = "<|semantic:{i}|>"
_SPECIALS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "<|pad|>", "<|phoneme_start|>", "<|phoneme_end|>",
             "<|text|>", "<|voice|>", "<|interleave|>", "<|audio_start|>", "<|audio_end|>", "<|audio_pad|>"]
_SPECIAL_RE = re.compile(r"(<\|[^<>|]+\|>)")


class FishFallbackTokenizer:
    """UTF-8 bytes at [3, 259); specials from 151643 (or lower, for small test vocabularies);
    speakers 0..22; then the contiguous semantic tokens (from 151678 at full size)."""

    SPECIAL_BASE = 151643
    NUM_SPEAKERS = 23

    def __init__(self, vocab_size: int = 155776, codebook_size: int = 4096, offset: int = 3):
        self.vocab_size = vocab_size
        self.offset = offset
        self._tok2id: dict[str, int] = {}
        nid = min(self.SPECIAL_BASE, vocab_size - codebook_size - len(_SPECIALS) - self.NUM_SPEAKERS)
        if nid < offset + 256:
            raise ValueError("vocabulary too small for bytes, special and semantic tokens")
        for s in _SPECIALS:
            self._tok2id[s] = nid
            nid += 1
        for i in range(self.NUM_SPEAKERS):
            self._tok2id[f"<|speaker:{i}|>"] = nid
            nid += 1
        self.semantic_begin_id = nid
        self.codebook_size = codebook_size
        self._id2tok = {v: k for k, v in self._tok2id.items()}
        if nid + codebook_size > vocab_size:
            raise ValueError("vocabulary too small for the semantic tokens")
        self.eos_token_id = self._tok2id[IM_END]

    def convert_tokens_to_ids(self, token):
        if isinstance(token, (list, tuple)):
            return [self.convert_tokens_to_ids(t) for t in token]
        m = re.fullmatch(r"<\|semantic:(\d+)\|>", token)
        if m:
            return self.semantic_begin_id + int(m.group(1))
        return self._tok2id[token]

    def encode(self, text: str, add_special_tokens: bool = True) -> list[int]:
        ids: list[int] = []
        for piece in _SPECIAL_RE.split(text):
            if not piece:
                continue
            if _SPECIAL_RE.fullmatch(piece):
                try:
                    ids.append(self.convert_tokens_to_ids(piece))
                    continue
                except KeyError:
                    pass
            ids.extend(b + self.offset for b in piece.encode("utf-8"))
        return ids

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        out, buf = [], bytearray()
        for i in ids:
            i = int(i)
            if self.offset <= i < self.offset + 256:
                buf.append(i - self.offset)
                continue
            if buf:
                out.append(buf.decode("utf-8", errors="replace"))
                buf = bytearray()
            if not skip_special_tokens:
                if self.semantic_begin_id <= i < self.semantic_begin_id + self.codebook_size:
                    out.append(SEMANTIC.format(i=i - self.semantic_begin_id))
                else:
                    out.append(self._id2tok.get(i, f"<{i}>"))
        if buf:
            out.append(buf.decode("utf-8", errors="replace"))
        return "".join(out)


def load_s2pro_tokenizer(model_path: str | None, vocab_size: int = 155776, codebook_size: int = 4096):
    if model_path and os.path.isdir(model_path) and os.path.exists(os.path.join(model_path, "tokenizer.json")):
        from transformers import PreTrainedTokenizerFast

        return PreTrainedTokenizerFast.from_pretrained(model_path)
    return FishFallbackTokenizer(vocab_size, codebook_size)


@dataclass
class Reference:
    """A voice-cloning reference: its transcript and its DAC codes [num_codebooks, frames]."""

    text: str = ""
    vq_codes: torch.Tensor | None = None


@dataclass
class S2ProPrompt:
    ids: list[int]
    vq_mask: list[bool]
    vq_codes: torch.Tensor          # int32 [n_vq, num_codebooks]

    def code_rows(self) -> torch.Tensor:
        """int32 [len(ids)]: row of vq_codes per position, -1 for text."""
        m = torch.tensor(self.vq_mask, dtype=torch.bool)
        r = torch.full((len(self.ids),), -1, dtype=torch.int32)
        r[m] = torch.arange(int(m.sum()), dtype=torch.int32)
        return r


class S2ProPromptBuilder:
    def __init__(self, tokenizer, num_codebooks: int = 10):
        self.tok = tokenizer
        self.num_codebooks = num_codebooks

    @property
    def im_end_id(self) -> int:
        return self.tok.convert_tokens_to_ids(IM_END)

    @property
    def semantic_begin_id(self) -> int:
        return self.tok.convert_tokens_to_ids(SEMANTIC.format(i=0))

    def build(self, text: str, references: list[Reference] | None = None, speaker: int | str = 0) -> S2ProPrompt:
        ids: list[int] = []
        mask: list[bool] = []
        codes: list[torch.Tensor] = []

        def add_text(s: str):
            t = self.tok.encode(s)
            ids.extend(t)
            mask.extend([False] * len(t))

        if references:
            add_text(f"{IM_START}system\n")
            add_text("convert the provided text to speech reference to the following:\n\nText:\n")
            for ref in references:
                if ref.text:
                    add_text(f"<|speaker:{speaker}|>{ref.text}")
            add_text("\n\nSpeech:\n")
            ref_codes = [torch.as_tensor(r.vq_codes) for r in references if r.vq_codes is not None]
            if ref_codes:
                c = torch.cat(ref_codes, dim=1).to(torch.int32)  # [num_codebooks, frames]
                sem = [SEMANTIC.format(i=int(i)) for i in c[0].tolist()]
                ids.extend(self.tok.convert_tokens_to_ids(sem))
                mask.extend([True] * c.shape[1])
                codes.append(c.t().contiguous())
            add_text(f"{IM_END}\n")
        add_text(f"{IM_START}user\n")
        add_text(f"<|speaker:{speaker}|>{text}")
        add_text(f"{IM_END}\n")
        add_text(f"{IM_START}assistant\n{VOICE}")
        vq = torch.cat(codes, 0) if codes else torch.zeros(0, self.num_codebooks, dtype=torch.int32)
        return S2ProPrompt(ids, mask, vq)
