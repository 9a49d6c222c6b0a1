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
