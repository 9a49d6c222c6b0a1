"""Pipeline configuration of Ming-Omni text output:
preprocessing -> audio_encoder -> mm_aggregate -> thinker -> decode
(stage names and routing as in sglang_omni/models/ming_omni/config.py:25-105)."""
from __future__ import annotations

from typing import ClassVar

from pydantic import Field

from ...config.schema import ExecutorConfig, InputHandlerConfig, PipelineConfig, StageConfig

_S = "sglang_omni_b200.models.ming_omni.pipeline.stages"
_N = "sglang_omni_b200.models.ming_omni.pipeline.next_stage"


def ming_stages(overrides=None, device="cuda:0", max_batch=64, max_context=8192):
    ov = {"overrides": overrides} if overrides else {}
    return [
        StageConfig(name="preprocessing", executor=ExecutorConfig(factory=f"{_S}.create_preprocessing_executor",
                                                                   args=dict(ov)),
                    get_next=f"{_N}.preprocessing_next"),
        StageConfig(name="audio_encoder", executor=ExecutorConfig(factory=f"{_S}.create_audio_encoder_executor",
                                                                   args={"device": device, **ov}),
                    get_next=f"{_N}.encoder_next"),
        StageConfig(name="mm_aggregate", executor=ExecutorConfig(factory=f"{_S}.create_aggregate_executor"),
                    get_next=f"{_N}.aggregate_next",
                    input_handler=InputHandlerConfig(type="aggregated", sources=["preprocessing", "audio_encoder"],
                                                     merge_fn="sglang_omni_b200.models.ming_omni.pipeline.merge."
                                                              "merge_for_thinker")),
        StageConfig(name="thinker", executor=ExecutorConfig(factory=f"{_S}.create_thinker_executor",
                                                             args={"device": device, "max_batch": max_batch,
                                                                   "max_context": max_context, **ov}),
                    get_next=f"{_N}.thinker_next"),
        StageConfig(name="decode", executor=ExecutorConfig(factory=f"{_S}.create_decode_executor"),
                    get_next=f"{_N}.decode_next"),
    ]


class MingOmniPipelineConfig(PipelineConfig):
    architecture: ClassVar[str] = "BailingMM2NativeForConditionalGeneration"
    entry_stage: str = "preprocessing"
    stages: list[StageConfig] = Field(default_factory=lambda: ming_stages())
    terminal_stages: list[str] = Field(default_factory=lambda: ["decode"])


EntryClass = MingOmniPipelineConfig
