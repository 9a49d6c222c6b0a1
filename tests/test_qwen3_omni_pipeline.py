"""Qwen3-Omni speech pipeline end to end on CPU with tiny random models:
audio in -> audio encoder -> thinker (text deltas) -> talker + code predictor
-> code2wav (audio chunks), multi-terminal result, through the OpenAI API."""
import asyncio
import json

import httpx
import pytest
import numpy as np
import torch

from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
from sglang_omni_b200.config import PipelineRunner, compile_pipeline
from sglang_omni_b200.models.qwen3_omni.config import Qwen3OmniSpeechPipelineConfig, text_stages
from sglang_omni_b200.serve.openai_api import create_app

TINY = {
    "thinker": {"num_layers": 2, "hidden_size": 64, "num_heads": 4, "num_kv_heads": 2, "head_dim": 32,
                "num_experts": 8, "topk": 2, "moe_intermediate_size": 32, "mrope_section": [6, 5, 5],
                "dtype": torch.float32},
    "talker": {"num_layers": 2, "hidden_size": 64, "num_heads": 4, "num_kv_heads": 2, "head_dim": 32,
               "num_experts": 8, "topk": 2, "moe_intermediate_size": 32, "shared_expert_intermediate_size": 32,
               "intermediate_size": 64, "mrope_section": [6, 5, 5], "dtype": torch.float32},
    "code_predictor": {"num_layers": 1, "hidden_size": 64, "num_heads": 4, "num_kv_heads": 2, "head_dim": 32,
                       "intermediate_size": 64, "dtype": torch.float32},
    "audio": {"encoder_layers": 1, "encoder_attention_heads": 2, "encoder_ffn_dim": 64, "d_model": 64,
              "downsample_hidden_size": 8, "dtype": torch.float32},
    "code2wav": {"codebook_size": 2048, "hidden_size": 64, "num_heads": 4, "num_kv_heads": 4,
                 "intermediate_size": 64, "num_layers": 1, "upsample_rates": (2, 2), "upsampling_ratios": (2,),
                 "decoder_dim": 32, "dtype": torch.float32},
}


def _cfg():
    return Qwen3OmniSpeechPipelineConfig(model_path="random", stages=text_stages(
        overrides=TINY, device="cpu", max_batch=4, max_context=1024, speech=True, tail_frames=12))


def test_speech_pipeline_cpu_end_to_end():
    async def main():
        coord, stages = compile_pipeline(_cfg())
        async with PipelineRunner(coord, stages):
            client = Client(coord)
            audio = (np.random.default_rng(0).standard_normal(16000 * 2) * 0.1).astype(np.float32)
            req = GenerateRequest(prompt="hello", audios=[audio], max_tokens=6,
                                  sampling=SamplingParams(temperature=0.0, ignore_eos=True),
                                  output_modalities=["text", "audio"], stream=True)
            text_chunks, audio_chunks, final = [], [], None
            async for ch in client.generate(req):
                if ch.finish_reason is not None:
                    final = ch
                elif ch.modality == "audio":
                    audio_chunks.append(ch.audio_data)
                else:
                    text_chunks.append(ch)
            assert len([c for c in text_chunks if c.token_ids]) == 6
            assert final is not None
            assert len(audio_chunks) >= 1
            assert final.audio_data is not None and len(final.audio_data) > 0

    asyncio.run(main())


def test_speech_pipeline_openai_sse_audio():
    async def main():
        coord, stages = compile_pipeline(_cfg())
        async with PipelineRunner(coord, stages):
            app = create_app(Client(coord), "qwen3-omni")
            async with httpx.AsyncClient(transport=httpx.ASGITransport(app=app), base_url="http://t") as http:
                body = {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 5, "temperature": 0.0,
                        "ignore_eos": True, "stream": True, "modalities": ["text", "audio"]}
                r = await http.post("/v1/chat/completions", json=body, timeout=120)
                events = [json.loads(ln[6:]) for ln in r.text.splitlines()
                          if ln.startswith("data: ") and ln != "data: [DONE]"]
                kinds = {("audio" if e["choices"][0]["delta"].get("audio") else "text") for e in events
                         if e.get("choices")}
                assert "audio" in kinds and "text" in kinds
                assert events[-1]["choices"][0]["finish_reason"] is not None

    asyncio.run(main())


GPU_TINY = {
    "thinker": {"num_layers": 2, "hidden_size": 256, "num_heads": 4, "num_kv_heads": 2, "head_dim": 64,
                "num_experts": 8, "topk": 2, "moe_intermediate_size": 128, "mrope_section": [12, 10, 10]},
    "talker": {"num_layers": 2, "hidden_size": 256, "num_heads": 4, "num_kv_heads": 2, "head_dim": 64,
               "num_experts": 8, "topk": 2, "moe_intermediate_size": 128, "shared_expert_intermediate_size": 128,
               "intermediate_size": 256, "mrope_section": [12, 10, 10]},
    "code_predictor": {"num_layers": 2, "hidden_size": 256, "num_heads": 4, "num_kv_heads": 2, "head_dim": 64,
                       "intermediate_size": 256},
    "audio": {"encoder_layers": 2, "encoder_attention_heads": 4, "encoder_ffn_dim": 512, "d_model": 256,
              "downsample_hidden_size": 64},
    "code2wav": {"hidden_size": 256, "num_heads": 4, "num_kv_heads": 4, "intermediate_size": 512, "num_layers": 2,
                 "upsample_rates": (4, 2), "upsampling_ratios": (2,), "decoder_dim": 256},
}


@pytest.mark.gpu
def test_speech_pipeline_gpu_end_to_end():
    async def main():
        cfg = Qwen3OmniSpeechPipelineConfig(model_path="random", stages=text_stages(
            overrides=GPU_TINY, device="cuda:0", max_batch=8, max_context=2048, speech=True, tail_frames=12))
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            client = Client(coord)
            audio = (np.random.default_rng(0).standard_normal(16000 * 3) * 0.1).astype(np.float32)

            async def one(i):
                req = GenerateRequest(prompt=f"hello {i}", audios=[audio], max_tokens=16,
                                      sampling=SamplingParams(temperature=0.0, ignore_eos=True),
                                      output_modalities=["text", "audio"], stream=True)
                n_text, n_audio, final = 0, 0, None
                async for ch in client.generate(req):
                    if ch.finish_reason is not None:
                        final = ch
                    elif ch.modality == "audio":
                        n_audio += 1
                    elif ch.token_ids:
                        n_text += 1
                return n_text, n_audio, final

            outs = await asyncio.gather(*[one(i) for i in range(4)])
            for n_text, n_audio, final in outs:
                assert n_text == 16 and n_audio >= 1
                assert final.audio_data is not None and len(final.audio_data) > 0

    asyncio.run(main())


def test_image_text_pipeline_batched_encoder_cpu():
    """Image + text -> text: requests with and without images arrive together; the image
    encoder stage runs the gathered images in one forward and splits the outputs back."""
    from sglang_omni_b200.models.qwen3_omni.config import Qwen3OmniPipelineConfig

    ov = dict(TINY, vision={"depth": 2, "hidden_size": 32, "num_heads": 2, "intermediate_size": 64,
                            "patch_size": 4, "out_hidden_size": 64, "num_position_embeddings": 64,
                            "deepstack_visual_indexes": [0], "dtype": torch.float32})
    cfg = Qwen3OmniPipelineConfig(model_path="random", stages=text_stages(overrides=ov, device="cpu", max_batch=4,
                                                                           max_context=1024))

    async def main():
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            client = Client(coord)
            rng = np.random.default_rng(1)
            imgs = [rng.integers(0, 256, (16, 24, 3), dtype=np.uint8), rng.integers(0, 256, (8, 8, 3), dtype=np.uint8)]

            async def one(req):
                last = None
                async for ch in client.generate(req):
                    last = ch
                return last

            reqs = [GenerateRequest(prompt="what is this", images=[imgs[0]], max_tokens=4, stream=False,
                                    sampling=SamplingParams(temperature=0.0, ignore_eos=True)),
                    GenerateRequest(prompt="and this", images=[imgs[1], imgs[0]], max_tokens=3, stream=False,
                                    sampling=SamplingParams(temperature=0.0, ignore_eos=True)),
                    GenerateRequest(prompt="text only", max_tokens=5, stream=False,
                                    sampling=SamplingParams(temperature=0.0, ignore_eos=True))]
            return await asyncio.gather(*[one(r) for r in reqs])

    outs = asyncio.run(main())
    assert [len(o.token_ids) for o in outs] == [4, 3, 5]


def _reference_speech_yaml(tmp_path):
    """The reference's 9-stage speech layout (sglang_omni/models/qwen3_omni/config.py:104-221)
    as YAML, with its factory / routing paths and arguments; only the tiny-model overrides and
    CPU devices are added for this test."""
    import yaml

    S = "sglang_omni.models.qwen3_omni.pipeline.stages"
    N = "sglang_omni.models.qwen3_omni.pipeline.next_stage"
    C = "sglang_omni.models.qwen3_omni.components"
    ov = {"overrides": {k: {a: ("float32" if b is torch.float32 else b) for a, b in v.items()}
                        for k, v in TINY.items()}}

    def stage(name, factory, args, nxt, stream_to=(), **extra):
        d = {"name": name, "executor": {"factory": factory, "args": args}, "get_next": f"{N}.{nxt}",
             "relay": {"device": "cpu"}, "stream_to": [{"to_stage": t, "bootstrap": b} for t, b in stream_to]}
        d.update(extra)
        return d

    cfg = {
        "model_path": "random", "entry_stage": "preprocessing", "terminal_stages": ["decode", "code2wav"],
        "gpu_placement": {"thinker": 0, "talker_ar": 1, "code_predictor": 1, "code2wav": 1},
        "stages": [
            stage("preprocessing", f"{S}.create_preprocessing_executor", dict(ov), "preprocessing_next"),
            stage("image_encoder", f"{S}.create_image_encoder_executor", {"device": "cpu", "dtype": None, **ov},
                  "encoder_next"),
            stage("audio_encoder", f"{S}.create_audio_encoder_executor", {"device": "cpu", "dtype": None, **ov},
                  "encoder_next"),
            stage("mm_aggregate", f"{S}.create_aggregate_executor", {}, "aggregate_next",
                  input_handler={"type": "aggregated", "sources": ["preprocessing", "image_encoder", "audio_encoder"],
                                 "merge_fn": "sglang_omni.models.qwen3_omni.pipeline.merge.merge_for_thinker"}),
            stage("thinker", f"{S}.create_sglang_thinker_executor_from_config",
                  {"thinker_max_seq_len": 1024, "speech_enabled": True, "device": "cpu", "max_batch": 4, **ov},
                  "thinker_next_speech", stream_to=[("talker_ar", True)]),
            stage("decode", f"{S}.create_decode_executor", {}, "decode_next"),
            stage("talker_ar", f"{S}.create_talker_ar_executor_from_config",
                  {"talker_max_seq_len": 1024, "speech_enabled": True, "feedback_enabled": True, "device": "cpu",
                   "max_streams": 4, "tail_frames": 12, **ov}, "talker_ar_next", stream_to=[("code_predictor", True)]),
            stage("code_predictor", f"{C}.code_predictor_executor.create_code_predictor_executor_from_config",
                  {"code_predictor_max_seq_len": 256}, "code_predictor_next",
                  stream_to=[("code2wav", True), ("talker_ar", False)]),
            stage("code2wav", f"{C}.code2wav_executor.create_code2wav_executor", {"device": "cpu", **ov},
                  "code2wav_next"),
        ],
    }
    p = tmp_path / "qwen3_omni_speech_reference_layout.yaml"
    p.write_text(yaml.safe_dump(cfg, sort_keys=False))
    return p


@pytest.mark.parametrize("fast_lanes", [True, False])
def test_reference_layout_yaml_runs(tmp_path, monkeypatch, fast_lanes):
    """A config in the reference's 9-stage layout compiles and serves a speech request."""
    from sglang_omni_b200.config.manager import ConfigManager
    from sglang_omni_b200.pipeline import fastlane

    if not fast_lanes:   # every hop over the relay, as between stage processes
        monkeypatch.setattr(fastlane, "get", lambda stage: None)
    cfg = ConfigManager.from_file(str(_reference_speech_yaml(tmp_path)))
    assert [s.name for s in cfg.stages][-3:] == ["talker_ar", "code_predictor", "code2wav"]

    async def main():
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            client = Client(coord)
            audio = (np.random.default_rng(2).standard_normal(16000) * 0.1).astype(np.float32)
            req = GenerateRequest(prompt="hi", audios=[audio], max_tokens=5,
                                  sampling=SamplingParams(temperature=0.0, ignore_eos=True),
                                  output_modalities=["text", "audio"], stream=True)
            text, audio_chunks, final = [], [], None
            async for ch in client.generate(req):
                if ch.finish_reason is not None:
                    final = ch
                elif ch.modality == "audio":
                    audio_chunks.append(ch)
                elif ch.token_ids:
                    text += ch.token_ids
            assert len(text) == 5 and audio_chunks and final is not None

    asyncio.run(main())
