"""Qwen3-Omni pipeline configurations (text and speech variants).

Stage graph and names follow sglang_omni/models/qwen3_omni/config.py:29-229:
  text:   preprocessing -> {image_encoder, audio_encoder, mm_aggregate} ->
          mm_aggregate (aggregated fan-in) -> thinker -> decode
  speech: + thinker streams to talker_ar, talker_ar streams codes to code2wav;
          terminal stages [decode, code2wav]; default placement keeps every
          speech stage on one GPU (the talker <-> code-predictor loop is
          in-graph), ``gpu_placement`` may move stages to other GPUs.
Executor args accept ``overrides`` (architecture shrinking for tests) and the
engine sizes (max_batch, max_context, ...).
"""
from __future__ import annotations

from typing import ClassVar

from pydantic import Field

from ...config.schema import (ExecutorConfig, InputHandlerConfig, PipelineConfig, StageConfig,
                              StreamTargetConfig)

_S = "sglang_omni_b200.models.qwen3_omni.pipeline.stages"
_N = "sglang_omni_b200.models.qwen3_omni.pipeline.next_stage"


def text_stages(overrides=None, device="cuda:0", max_batch=64, max_context=4096, speech=False, tail_frames=50,
                first_chunk=4, thinker_parallel: dict | None = None, encoder_cache: int = 64):
    """``first_chunk``: frames of the first Code2Wav chunk (later chunks are 10 frames of 80 ms);
    ``thinker_parallel``: ``tp_size`` / ``ep_size`` / ``gpus`` of a thinker rank group;
    ``encoder_cache``: encoder outputs each tower keeps by media content key (0: every request's
    media is encoded and preprocessing computes no keys)."""
    ov = {"overrides": overrides} if overrides else {}
    cache = {"cache_size": int(encoder_cache)}
    thinker_args = {"device": device, "max_batch": max_batch, "max_context": max_context, **ov,
                    **(thinker_parallel or {})}
    if speech:
        thinker_args["speech_target"] = "talker_ar"
    stages = [
        StageConfig(name="preprocessing", executor=ExecutorConfig(factory=f"{_S}.create_preprocessing_executor",
                                                                   args={**ov, "cache_keys": encoder_cache > 0}),
                    get_next=f"{_N}.preprocessing_next"),
        StageConfig(name="image_encoder", executor=ExecutorConfig(factory=f"{_S}.create_image_encoder_executor",
                                                                   args={"device": device, **ov, **cache}),
                    get_next=f"{_N}.encoder_next"),
        StageConfig(name="audio_encoder", executor=ExecutorConfig(factory=f"{_S}.create_audio_encoder_executor",
                                                                   args={"device": device, **ov, **cache}),
                    get_next=f"{_N}.encoder_next"),
        StageConfig(name="mm_aggregate", executor=ExecutorConfig(factory=f"{_S}.create_aggregate_executor"),
                    get_next=f"{_N}.aggregate_next",
                    input_handler=InputHandlerConfig(type="aggregated",
                                                     sources=["preprocessing", "image_encoder", "audio_encoder"],
                                                     merge_fn="sglang_omni_b200.models.qwen3_omni.pipeline.merge.merge_for_thinker")),
        StageConfig(name="thinker", executor=ExecutorConfig(factory=f"{_S}.create_thinker_executor",
                                                             args=thinker_args),
                    get_next=f"{_N}.thinker_next",
                    stream_to=[StreamTargetConfig(to_stage="talker_ar", bootstrap=True)] if speech else []),
        StageConfig(name="decode", executor=ExecutorConfig(factory=f"{_S}.create_decode_executor"),
                    get_next=f"{_N}.decode_next"),
    ]
    if speech:
        stages += [
            StageConfig(name="talker_ar", executor=ExecutorConfig(factory=f"{_S}.create_talker_executor",
                                                                   args={"device": device, "max_streams": max_batch,
                                                                         "tail_frames": tail_frames, **ov}),
                        get_next=f"{_N}.talker_next",
                        stream_to=[StreamTargetConfig(to_stage="code2wav", bootstrap=True)]),
            StageConfig(name="code2wav", executor=ExecutorConfig(factory=f"{_S}.create_code2wav_executor",
                                                                  args={"device": device, "first_chunk": first_chunk,
                                                                        **ov}),
                        get_next=f"{_N}.code2wav_next"),
        ]
    return stages


class Qwen3OmniPipelineConfig(PipelineConfig):
    architecture: ClassVar[str] = "Qwen3OmniMoeForConditionalGeneration"
    entry_stage: str = "preprocessing"
    stages: list[StageConfig] = Field(default_factory=lambda: text_stages())
    terminal_stages: list[str] = Field(default_factory=lambda: ["decode"])


class Qwen3OmniSpeechPipelineConfig(PipelineConfig):
    architecture: ClassVar[str] = "Qwen3OmniMoeForConditionalGeneration"
    entry_stage: str = "preprocessing"
    stages: list[StageConfig] = Field(default_factory=lambda: text_stages(speech=True))
    terminal_stages: list[str] = Field(default_factory=lambda: ["decode", "code2wav"])


Qwen3OmniSpeechPipelineConfig.Variants = {"text": Qwen3OmniPipelineConfig, "speech": Qwen3OmniSpeechPipelineConfig}
EntryClass = Qwen3OmniSpeechPipelineConfig
