"""State of one autoregressive request inside the paged engine."""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any, Callable

import torch

from ...sampling_params import SamplingParams


@dataclass
class ARRequest:
    rid: str
    prompt_ids: list[int]
    sampling: SamplingParams = field(default_factory=SamplingParams)
    max_new_tokens: int = 128
    eos_token_ids: tuple = ()
    # multimodal / projected prefill inputs
    input_embeds: torch.Tensor | None = None       # [L, H] replaces the token embedding
    mm_index: torch.Tensor | None = None           # [L] row of mm_embeds or -1
    mm_embeds: torch.Tensor | None = None
    mrope_positions: torch.Tensor | None = None    # [3, L] prompt positions (M-RoPE)
    mrope_delta: int = 0                           # decode position = cache length + delta
    deepstack: list | None = None                  # per layer [L_vis, H] embeds, with ds_positions
    ds_positions: torch.Tensor | None = None
    capture_layers: tuple = ()                     # hidden states to emit per generated token
    capture_prompt_layer: int | None = None        # keep this layer's prompt rows in extra['prompt_hidden']
    on_token: Callable[["ARRequest", int, dict], None] | None = None
    extra: dict[str, Any] = field(default_factory=dict)
    # engine state
    slot: int = -1
    pages: list = field(default_factory=list)
    num_cached: int = 0          # tokens whose K/V are in the cache
    output_ids: list[int] = field(default_factory=list)
    finished: bool = False
    finish_reason: str | None = None
    aborted: bool = False
    arrival: float = field(default_factory=time.perf_counter)
    first_token_time: float | None = None
    finish_time: float | None = None
    scheduled_decodes: int = 0   # decode steps launched since the last (re)prefill
    folded: int = 0              # generated tokens re-prefilled after a KV retraction
    prefix_nodes: list = field(default_factory=list)  # prefix-cache nodes this request holds (pages[:n])
    cached_tokens: int = 0       # prompt tokens served from the prefix cache

    @property
    def prompt_len(self) -> int:
        """Length of the sequence the next prefill covers (prompt + folded outputs)."""
        return len(self.prompt_ids) + self.folded

    def prefill_ids(self, start: int, end: int) -> list[int]:
        n = len(self.prompt_ids)
        if end <= n:
            return self.prompt_ids[start:end]
        return list(self.prompt_ids[start:n]) + self.output_ids[max(0, start - n):end - n] if start < n \
            else self.output_ids[start - n:end - n]

    @property
    def prefill_done(self) -> bool:
        return self.num_cached >= self.prompt_len

    @property
    def total_len(self) -> int:
        return self.prompt_len + len(self.output_ids)

    def check_stop(self, token: int) -> bool:
        if len(self.output_ids) >= self.max_new_tokens:
            self.finish_reason = "length"
            return True
        if not self.sampling.ignore_eos and (token in self.eos_token_ids or token in self.sampling.stop_token_ids):
            self.finish_reason = "stop"
            return True
        return False
