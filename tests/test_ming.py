"""Ming-Omni: Whisper audio tower vs an fp32 oracle, the chat layout with audio
patches, and the 5-stage text pipeline end to end (tiny random models)."""
import asyncio
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from sglang_omni_b200.models.ming_omni.audio_encoder import MingAudioEncoder, sinusoids
from sglang_omni_b200.models.ming_omni.hf_config import AUDIO_PATCH, WhisperConfig, audio_tokens

W_TINY = dict(n_mels=128, n_ctx=400, n_state=128, n_head=2, n_layer=2, out_dim=64)
TINY = {"llm": {"vocab_size": 1024, "hidden_size": 64, "num_layers": 2, "num_heads": 4, "num_kv_heads": 2,
                "head_dim": 64, "rotary_dim": 32, "intermediate_size": 128, "num_experts": 64, "topk": 4,
                "moe_intermediate_size": 32, "shared_expert_intermediate_size": 32, "n_group": 2, "topk_group": 1},
        "whisper": W_TINY}


def whisper_reference(enc: MingAudioEncoder, mel: torch.Tensor) -> torch.Tensor:
    """Plain fp32 restatement from the module's parameters (conv weights re-viewed as [O, I, K])."""
    cfg = enc.cfg
    D, M = cfg.n_state, cfg.n_mels
    f = lambda t: t.float()  # noqa: E731
    w1 = f(enc.conv1_w).view(D, 3, M).permute(0, 2, 1)
    w2 = f(enc.conv2_w).view(D, 3, D).permute(0, 2, 1)
    x = F.gelu(F.conv1d(mel[None].float(), w1, f(enc.conv1_b), padding=1))
    x = F.gelu(F.conv1d(x, w2, f(enc.conv2_b), stride=2, padding=1))[0].t()
    x = x + f(enc.pos[: x.shape[0]])
    hd = D // cfg.n_head
    for B in enc.blocks:
        n = F.layer_norm(x, (D,), f(B.ln1_w), f(B.ln1_b), 1e-5)
        q, k, v = (n @ f(B.qkv_w).t() + f(B.qkv_b)).split(D, -1)
        q, k, v = (t.view(-1, cfg.n_head, hd).transpose(0, 1) for t in (q, k, v))
        a = F.scaled_dot_product_attention(q, k, v).transpose(0, 1).reshape(-1, D)
        x = x + a @ f(B.o_w).t() + f(B.o_b)
        n = F.layer_norm(x, (D,), f(B.ln2_w), f(B.ln2_b), 1e-5)
        x = x + F.gelu(n @ f(B.fc1_w).t() + f(B.fc1_b)) @ f(B.fc2_w).t() + f(B.fc2_b)
    x = F.layer_norm(x, (D,), f(enc.ln_post_w), f(enc.ln_post_b), 1e-5)
    k = cfg.ds_kernel_size
    wp = f(enc.proj_w).view(cfg.out_dim, k, D).permute(0, 2, 1)
    y = F.conv1d(x.t()[None], wp, f(enc.proj_b), stride=cfg.ds_stride, padding=k // 2)[0].t()
    for L in enc.mlp:
        y = F.gelu(y) @ f(L.w).t() + f(L.b)
    return F.normalize(y, dim=-1)


def test_sinusoids_definition():
    s = sinusoids(10, 8)
    inc = math.log(10000) / 3
    assert torch.allclose(s[3, 1], torch.tensor(math.sin(3 * math.exp(-inc))))
    assert torch.allclose(s[3, 5], torch.tensor(math.cos(3 * math.exp(-inc))))


def test_audio_encoder_matches_reference_cpu():
    torch.manual_seed(0)
    enc = MingAudioEncoder(WhisperConfig(**W_TINY), dtype=torch.float32).random_init_(seed=1, std=0.05)
    mels = [torch.randn(128, 37), torch.randn(128, 100)]
    outs = enc(mels)
    for m, o in zip(mels, outs):
        ref = whisper_reference(enc, m)
        assert o.shape[0] == audio_tokens(m.shape[1], enc.cfg) == enc.output_length(m.shape[1])
        torch.testing.assert_close(o.float(), ref, atol=2e-4, rtol=2e-4)


def test_prompt_layout_audio_patches():
    from sglang_omni_b200.models.ming_omni import loader
    from sglang_omni_b200.models.ming_omni.pipeline.stages import build_prompt

    tok = loader.get_tokenizer("random", TINY)
    ids, spans = build_prompt(tok, None, "what is this?", [5, 3])
    assert [e - s for s, e in spans] == [5, 3]
    text = tok.decode(ids, skip_special_tokens=False)
    assert text.startswith("<role>SYSTEM</role>")
    assert "<role>HUMAN</role><audio>" + AUDIO_PATCH * 5 + "</audio><audio>" in text
    assert text.endswith("what is this?<|role_end|><role>ASSISTANT</role>")


def _pipeline(device):
    from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
    from sglang_omni_b200.config import PipelineRunner, compile_pipeline
    from sglang_omni_b200.models.ming_omni.config import MingOmniPipelineConfig, ming_stages

    cfg = MingOmniPipelineConfig(model_path="random", stages=ming_stages(overrides=TINY, device=device, max_batch=4,
                                                                         max_context=1024))

    async def main():
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            client = Client(coord)
            audio = (np.random.default_rng(0).standard_normal(16000) * 0.1).astype(np.float32)
            reqs = [GenerateRequest(prompt="Describe.", audios=[audio], max_tokens=6, stream=False,
                                    sampling=SamplingParams(temperature=0.0, ignore_eos=True)),
                    GenerateRequest(prompt="Hello", max_tokens=5, stream=False,
                                    sampling=SamplingParams(temperature=0.0, ignore_eos=True))]
            return await asyncio.gather(*[_final(client, r) for r in reqs])

    return asyncio.run(main())


async def _final(client, req):
    last = None
    async for ch in client.generate(req):
        last = ch
    return last


def test_ming_pipeline_cpu_end_to_end():
    outs = _pipeline("cpu")
    assert len(outs[0].token_ids) == 6 and len(outs[1].token_ids) == 5


@pytest.mark.gpu
def test_audio_encoder_gpu_matches_cpu():
    cpu = MingAudioEncoder(WhisperConfig(**W_TINY), dtype=torch.float32).random_init_(seed=2, std=0.05)
    gpu = MingAudioEncoder(WhisperConfig(**W_TINY), device="cuda")
    with torch.no_grad():
        for (_, a), (_, b) in zip(cpu.named_parameters(), gpu.named_parameters()):
            b.copy_(a.to(b.dtype))
    mels = [torch.randn(128, 64), torch.randn(128, 150)]
    for c, g in zip(cpu(mels), gpu([m.cuda() for m in mels])):
        assert float((g.float().cpu() - c).norm() / c.norm()) < 0.03


@pytest.mark.gpu
def test_ming_pipeline_gpu_end_to_end():
    outs = _pipeline("cuda:0")
    assert len(outs[0].token_ids) == 6 and len(outs[1].token_ids) == 5
