"""Pipeline configuration of FishAudio S2-Pro TTS: preprocessing -> tts_engine -> vocoder
(stage names, factories and routing as in sglang_omni/models/fishaudio_s2_pro/config.py:22-56)."""
from __future__ import annotations

from typing import ClassVar

from pydantic import Field

from ...config.schema import ExecutorConfig, PipelineConfig, RelayConfig, StageConfig

_S = "sglang_omni_b200.models.fishaudio_s2_pro.pipeline.stages"
_N = "sglang_omni_b200.models.fishaudio_s2_pro.pipeline.next_stage"


def s2pro_stages(overrides=None, device="cuda:0", max_new_tokens=2048, max_streams=64, max_context=4096,
                 stream_stride=5, stream_followup_stride=20):
    ov = {"overrides": overrides} if overrides else {}
    return [
        StageConfig(name="preprocessing", executor=ExecutorConfig(factory=f"{_S}.create_preprocessing_executor",
                                                                  args={**ov}),
                    get_next=f"{_N}.preprocessing_next", relay=RelayConfig(device="cpu")),
        StageConfig(name="tts_engine", executor=ExecutorConfig(
            factory=f"{_S}.create_tts_engine_executor",
            args={"device": device, "max_new_tokens": max_new_tokens, "max_streams": max_streams,
                  "max_context": max_context, "stream_stride": stream_stride,
                  "stream_followup_stride": stream_followup_stride, **ov}),
            get_next=f"{_N}.tts_engine_next", relay=RelayConfig(device="cpu")),
        StageConfig(name="vocoder", executor=ExecutorConfig(factory=f"{_S}.create_vocoder_executor",
                                                            args={"device": device, **ov}),
                    get_next=f"{_N}.vocoder_next", relay=RelayConfig(device="cpu")),
    ]


class S2ProPipelineConfig(PipelineConfig):
    architecture: ClassVar[str] = "FishQwen3OmniForCausalLM"
    entry_stage: str = "preprocessing"
    stages: list[StageConfig] = Field(default_factory=lambda: s2pro_stages())
    terminal_stages: list[str] = Field(default_factory=lambda: ["vocoder"])


EntryClass = S2ProPipelineConfig
