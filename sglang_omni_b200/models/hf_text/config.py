"""Text pipeline of a Hugging Face causal LM checkpoint: ``preprocessing`` (chat template /
tokenizer of the checkpoint, or the byte tokenizer when it ships none) -> ``decoder`` (the
converted model on the paged AR engine, streamed text).  Registered for the architectures in
``convert.SUPPORTED_ARCHITECTURES``, so ``sgl-omni serve --model-path <checkpoint dir>`` picks
it from the checkpoint's config.json, like the reference's two-stage Llama demo / OpenAI Llama
server (examples/run_two_stage_llama_demo.py, examples/run_openai_llama_server.py)."""
from __future__ import annotations

from typing import ClassVar

from pydantic import Field

from ...config.schema import ExecutorConfig, PipelineConfig, StageConfig
from .convert import SUPPORTED_ARCHITECTURES

_P = "sglang_omni_b200.models"


def hf_text_stages(device: str = "cuda:0", max_batch: int = 64, max_context: int = 4096,
                   max_prefill_tokens: int = 8192, use_graphs: bool = True) -> list[StageConfig]:
    return [
        StageConfig(name="preprocessing",
                    executor=ExecutorConfig(factory=f"{_P}.hf_text.config.create_hf_preprocessing_executor"),
                    get_next=f"{_P}.hf_text.config.to_decoder"),
        StageConfig(name="decoder",
                    executor=ExecutorConfig(factory=f"{_P}.hf_text.config.create_hf_decoder_executor",
                                            args={"device": device, "max_batch": max_batch,
                                                  "max_context": max_context,
                                                  "max_prefill_tokens": max_prefill_tokens,
                                                  "use_graphs": use_graphs}),
                    get_next=f"{_P}.common.text_stages.terminal"),
    ]


class HFTextPipelineConfig(PipelineConfig):
    architectures: ClassVar[list[str]] = list(SUPPORTED_ARCHITECTURES)
    entry_stage: str = "preprocessing"
    stages: list[StageConfig] = Field(default_factory=hf_text_stages)
    terminal_stages: list[str] = Field(default_factory=lambda: ["decoder"])


def to_decoder(request_id, payload):
    return "decoder"


def _vocab(model_path: str) -> int:
    import json
    import os

    with open(os.path.join(model_path, "config.json")) as f:
        return int(json.load(f)["vocab_size"])


def create_hf_preprocessing_executor(model_path: str = ""):
    from ..common.text_stages import create_text_preprocessing_executor

    return create_text_preprocessing_executor(model_path, _vocab(model_path))


def create_hf_decoder_executor(model_path: str = "", device: str = "cuda:0", max_batch: int = 64,
                               max_context: int = 4096, max_prefill_tokens: int = 8192, use_graphs: bool = True,
                               dtype: str | None = None, default_max_new_tokens: int = 256):
    import torch

    from ..common.ar_stage import create_ar_executor
    from ..common.tokenizer import load_tokenizer
    from .convert import decoder_from_hf, eos_token_ids

    dt = {"bf16": torch.bfloat16, "bfloat16": torch.bfloat16, "fp16": torch.float16, "float16": torch.float16,
          "fp32": torch.float32, "float32": torch.float32}.get(dtype) if dtype else None
    model = decoder_from_hf(model_path, device, dt, max_position=max_context)
    tok = load_tokenizer(model_path, model.cfg.vocab_size)
    return create_ar_executor(model, "decoder", tok, max_batch=max_batch, max_context=max_context,
                              max_prefill_tokens=max_prefill_tokens, use_graphs=use_graphs,
                              eos_token_ids=eos_token_ids(model_path), default_max_new_tokens=default_max_new_tokens)


EntryClass = HFTextPipelineConfig
