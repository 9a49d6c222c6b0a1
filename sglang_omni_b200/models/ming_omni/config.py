"""Pipeline configurations of Ming-Omni:
text output   preprocessing -> audio_encoder -> mm_aggregate -> thinker -> decode;
speech output the same, with the thinker fanning out to decode and talker
(stage names and routing as in sglang_omni/models/ming_omni/config.py:25-202)."""
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


def ming_speech_stages(overrides=None, device="cuda:0", talker_device=None, max_batch=64, max_context=8192,
                       max_streams=32):
    st = ming_stages(overrides, device, max_batch, max_context)
    for s in st:
        if s.name == "thinker":
            s.get_next = f"{_N}.thinker_next_speech"
    ov = {"overrides": overrides} if overrides else {}
    st.append(StageConfig(name="talker", executor=ExecutorConfig(
        factory=f"{_S}.create_talker_executor",
        args={"device": talker_device or device, "max_streams": max_streams, **ov}),
        get_next=f"{_N}.talker_next"))
    return st


class MingOmniSpeechPipelineConfig(PipelineConfig):
    """Text + speech output: the talker (own Qwen2 LM + CFM/DiT + AudioVAE) speaks the thinker's text."""
    architecture: ClassVar[str] = "BailingMM2NativeForConditionalGeneration"
    entry_stage: str = "preprocessing"
    stages: list[StageConfig] = Field(default_factory=lambda: ming_speech_stages())
    terminal_stages: list[str] = Field(default_factory=lambda: ["decode", "talker"])


EntryClass = MingOmniPipelineConfig
