"""Two-stage toy pipeline for plumbing tests without a GPU.

Stage 1 ``preprocessing`` is an identity stage; stage 2 ``decoder`` is a
Llama-style decoder (2 layers, hidden 64, 4 heads x 16, SiLU MLP 256, RMSNorm
eps 1e-6, RoPE theta 1e4, vocab 1000, fp32, N(0, 0.02) weights from seed 0)
served by the paged AR engine with streaming output.
"""
from __future__ import annotations

from typing import ClassVar

from pydantic import Field

from ...config.schema import ExecutorConfig, PipelineConfig, StageConfig

_P = "sglang_omni_b200.models"


def _stages():
    return [
        StageConfig(name="preprocessing",
                    executor=ExecutorConfig(factory=f"{_P}.common.text_stages.create_identity_executor"),
                    get_next=f"{_P}.toy.config.to_decoder"),
        StageConfig(name="decoder",
                    executor=ExecutorConfig(factory=f"{_P}.toy.config.create_toy_decoder_executor",
                                            args={"device": "cpu"}),
                    get_next=f"{_P}.common.text_stages.terminal"),
    ]


class ToyPipelineConfig(PipelineConfig):
    architecture: ClassVar[str] = "ToyLlamaForCausalLM"
    model_path: str = "toy"
    entry_stage: str = "preprocessing"
    stages: list[StageConfig] = Field(default_factory=_stages)
    terminal_stages: list[str] = Field(default_factory=lambda: ["decoder"])


def to_decoder(request_id, payload):
    return "decoder"


def toy_decoder_config():
    import torch

    from ..decoder import DecoderConfig

    return DecoderConfig(vocab_size=1000, hidden_size=64, num_layers=2, num_heads=4, num_kv_heads=4, head_dim=16,
                         intermediate_size=256, rms_norm_eps=1e-6, rope_theta=10000.0, qk_norm=False,
                         max_position=2048, dtype=torch.float32, name="toy_llama")


def build_toy_rank(args: dict, rank: int, world: int, device, group, mode: str):
    """A full copy of the toy decoder on every rank of a stage group (``replica`` / ``dp`` modes)."""
    from ..decoder import DecoderLM

    return DecoderLM(toy_decoder_config(), device=device).random_init_(seed=int(args.get("seed", 0)))


def create_toy_decoder_executor(device: str = "cpu", max_batch: int = 8, seed: int = 0, group_mode: str | None = None,
                                group_size: int = 1, group_tp: int = 1):
    """``group_mode`` ("replica" or "dp") with ``group_size`` > 1 serves the decoder with a stage
    rank group of that many processes (the plumbing of TP / EP stages, on CPU); ``group_tp`` > 1
    (``dp``) forms lock-step groups of that many ranks, the plumbing of TP x EP stages."""
    import torch

    from ..common.ar_stage import create_ar_executor
    from ..common.tokenizer import ByteTokenizer
    from ..decoder import DecoderLM

    common = dict(max_batch=max_batch, max_context=512, max_prefill_tokens=512, use_graphs=False,
                  default_max_new_tokens=16)
    if group_mode and group_size > 1:
        from ...parallel.rank_group import GroupSpec

        spec = GroupSpec(mode=group_mode, world=group_size, builder=f"{_P}.toy.config.build_toy_rank",
                         builder_args={"seed": seed}, report_timeout_s=60.0, tp=group_tp)
        return create_ar_executor(None, "decoder", ByteTokenizer(1000), rank_group=spec, **common)
    torch.manual_seed(seed)
    model = DecoderLM(toy_decoder_config(), device=device).random_init_(seed=seed)
    return create_ar_executor(model, "decoder", ByteTokenizer(1000), **common)


EntryClass = ToyPipelineConfig
