"""Ming-Omni talker (Qwen2 LM + CFM/DiT + aggregator) and AudioVAE decoder against
plain fp32 restatements of the math, the batched generator, and the speech pipeline."""
import asyncio
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from sglang_omni_b200.models.ming_omni.audio_vae import AudioVAEConfig, AudioVAEDecoder
from sglang_omni_b200.models.ming_omni.talker import (BlockStack, MingSpeechGenerator, MingTalker, MingTalkerConfig,
                                                      RowLayout, build_talker_prompt, cfm_timesteps, qwen2_config,
                                                      timestep_embedding)

LLM_TINY = dict(vocab_size=1024, hidden_size=64, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64,
                intermediate_size=128, max_position=4096)


def tiny_cfg(dtype=torch.float32):
    return MingTalkerConfig(llm=qwen2_config(dtype=dtype, **LLM_TINY), dit_hidden=96, dit_depth=2, dit_heads=4,
                            agg_hidden=72, agg_depth=2, agg_heads=4, patch_size=4, history_patch_size=8,
                            latent_dim=16, spk_dim=24, steps=10, dtype=dtype)


# ----------------------------------------------------------------------------- oracles
def rope_pairs(x, pos, theta=10000.0):
    """Interleaved-pair rotary embedding: pair (2i, 2i+1) turns by pos * theta^(-2i/d)."""
    d = x.shape[-1]
    inv = 1.0 / theta ** (torch.arange(0, d, 2).float() / d)
    ang = pos.float()[:, None] * inv[None, :]
    c, s = ang.cos(), ang.sin()
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x1 * c + x0 * s
    return out


def rms(x, w, eps=1e-6):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def stack_oracle(st: BlockStack, x, lens):
    """[sum lens, hidden] fp32, bidirectional attention inside each sequence."""
    f = lambda t: t.float()  # noqa: E731
    h, d, dk = st.heads, st.d, st.dk
    outs = []
    off = 0
    for n in lens:
        y = x[off:off + n].float()
        pos = torch.arange(n)
        for L in st.layers:
            a = rms(y, f(L.n1))
            qkv = a @ f(L.qkv).t() + f(L.qkv_b)
            q, k, v = (t.view(n, h, dk)[..., :d] for t in qkv.split(h * dk, -1))
            q = rope_pairs(q.transpose(0, 1), pos)
            k = rope_pairs(k.transpose(0, 1), pos)
            o = F.scaled_dot_product_attention(q, k, v.transpose(0, 1)).transpose(0, 1)   # [n, h, d]
            o = F.pad(o, (0, dk - d)).reshape(n, h * dk)
            y = y + o @ f(L.o).t() + f(L.o_b)
            m = rms(y, f(L.n2))
            y = y + F.gelu(m @ f(L.f1).t() + f(L.f1_b), approximate="tanh") @ f(L.f2).t() + f(L.f2_b)
        outs.append(y)
        off += n
    return torch.cat(outs, 0)


def velocity_oracle(t: MingTalker, x, tt, cond, his):
    f = lambda p: p.float()  # noqa: E731
    c = t.cfg
    te = timestep_embedding(tt, c.freq_embed_dim)
    te = F.silu(te @ f(t.t1).t() + f(t.t1_b)) @ f(t.t2).t() + f(t.t2_b)
    y = te + cond.float() @ f(t.c_emb).t() + f(t.c_emb_b)
    lat = torch.cat([his, x], 1).float() @ f(t.x_emb).t() + f(t.x_emb_b)
    seq = torch.cat([y[:, None], lat], 1)
    N, L, D = seq.shape
    h = stack_oracle(t.dit, seq.reshape(N * L, D), [L] * N).view(N, L, D)[:, -c.patch_size:]
    return rms(h, f(t.dit_norm)) @ f(t.dit_out).t() + f(t.dit_out_b)


def cfm_oracle(t: MingTalker, cond, his, noise, cfg_strength):
    ts = cfm_timesteps(t.cfg.steps)
    y = noise.float()
    z = torch.zeros_like(cond)
    for s in range(len(ts) - 1):
        tt = torch.full((cond.shape[0],), ts[s])
        vc = velocity_oracle(t, y, tt, cond, his)
        vn = velocity_oracle(t, y, tt, z, his)
        y = y + (vc + (vc - vn) * cfg_strength) * (ts[s + 1] - ts[s])
    return y


def aggregate_oracle(t: MingTalker, lat):
    f = lambda p: p.float()  # noqa: E731
    B, P, Z = lat.shape
    x = lat.float() @ f(t.a_x).t() + f(t.a_x_b)
    seq = torch.cat([f(t.a_cls).view(1, 1, -1).expand(B, 1, -1), x], 1)
    h = stack_oracle(t.agg, seq.reshape(B * (P + 1), -1), [P + 1] * B).view(B, P + 1, -1)[:, 0]
    return rms(h, f(t.agg_norm)) @ f(t.agg_out).t() + f(t.agg_out_b)


def istft_oracle(spec_re, spec_im, n_fft, hop):
    """'same'-padded ISTFT: irfft -> Hann window -> overlap-add -> / window envelope -> trim."""
    B, L, K = spec_re.shape
    win = torch.hann_window(n_fft, periodic=True, dtype=torch.float64)
    fr = torch.fft.irfft(torch.complex(spec_re.double(), spec_im.double()), n_fft, dim=-1) * win
    out_len = (L - 1) * hop + n_fft
    y = F.fold(fr.transpose(1, 2), (1, out_len), (1, n_fft), stride=(1, hop))[:, 0, 0]
    env = F.fold(win.square().expand(1, L, n_fft).transpose(1, 2), (1, out_len), (1, n_fft), stride=(1, hop))[0, 0, 0]
    pad = (n_fft - hop) // 2
    return (y[:, pad:-pad] / env[pad:-pad]).float()


# ----------------------------------------------------------------------------- CPU tier
def test_cfm_schedule():
    ts = cfm_timesteps(10)
    assert ts[0] == 0.0 and abs(ts[-1] - 1.0) < 1e-12
    raw = [0, 2, 4, 6, 8, 12, 16, 20, 24, 28, 32]
    for v, r in zip(ts, raw):
        assert abs(v - (1 - math.cos(math.pi / 2 * r / 32))) < 1e-12   # sway -1 warps t to 1 - cos(pi t / 2)
    assert all(b > a for a, b in zip(ts, ts[1:]))


def test_block_stack_padded_heads_cpu():
    torch.manual_seed(0)
    st = BlockStack(72, 2, 4, 4.0, "cpu", torch.float32)   # head 18 -> kernel head 64 (zero padded)
    st.random_init_(torch.Generator().manual_seed(1), 0.1)
    assert st.dk == 64
    lens = [5, 9]
    x = torch.randn(sum(lens), 72)
    lay = RowLayout(1, 1, "cpu")
    pos = torch.cat([torch.arange(n, dtype=torch.int32) for n in lens])
    cu = torch.tensor([0, 5, 14], dtype=torch.int32)
    y = st(x, pos, cu, lens)
    ref = stack_oracle(st, x, lens)
    assert float((y - ref).abs().max()) < 1e-4
    del lay


def test_dit_cfm_aggregator_cpu():
    torch.manual_seed(0)
    t = MingTalker(tiny_cfg()).random_init_(seed=3, std=0.1)
    c = t.cfg
    B = 3
    cond = torch.randn(B, c.llm.hidden_size)
    his = torch.randn(B, c.history_patch_size, c.latent_dim)
    x = torch.randn(B, c.patch_size, c.latent_dim)
    rows = RowLayout(B, 1 + c.history_patch_size + c.patch_size, "cpu")
    v = t.dit_velocity(x, torch.full((B,), 0.3), cond, his, rows)
    assert float((v - velocity_oracle(t, x, torch.full((B,), 0.3), cond, his)).abs().max()) < 1e-4
    rows2 = RowLayout(2 * B, 1 + c.history_patch_size + c.patch_size, "cpu")
    y = t.cfm_sample(cond, his, x, cfm_timesteps(c.steps), 2.0, rows2)
    assert float((y - cfm_oracle(t, cond, his, x, 2.0)).abs().max()) < 1e-3
    agg = t.aggregate(y, RowLayout(B, 1 + c.patch_size, "cpu"))
    assert float((agg - aggregate_oracle(t, y)).abs().max()) < 1e-4


def test_istft_head_matches_oracle_cpu():
    cfg = AudioVAEConfig(hop=40, hidden=64, layers=1, heads=1, kv_heads=1, intermediate=128, latent_dim=16,
                         dtype=torch.float32)
    vae = AudioVAEDecoder(cfg).random_init_(seed=1, std=0.05)
    h = torch.randn(2, 11, 64)
    y = vae.istft_head(h)
    K = cfg.n_fft // 2 + 1
    pred = h @ vae.head.float().t() + vae.head_b.float()
    mag = torch.exp(pred[..., :K]).clamp(max=1e2)
    ph = pred[..., K:]
    ref = istft_oracle(mag * torch.cos(ph), mag * torch.sin(ph), cfg.n_fft, cfg.hop)
    assert y.shape == (2, 11 * cfg.hop) == ref.shape
    assert float((y - ref).abs().max() / ref.abs().max()) < 1e-4


def test_vae_decode_shapes_and_streaming_cpu():
    cfg = AudioVAEConfig(hop=40, hidden=64, layers=2, heads=1, kv_heads=1, intermediate=128, latent_dim=16,
                         dtype=torch.float32)
    vae = AudioVAEDecoder(cfg).random_init_(seed=2, std=0.05)
    z = torch.randn(1, 9, 16)
    full = vae.decode(z)[0]
    assert full.shape == (9 * cfg.patch_size * cfg.hop,) and torch.isfinite(full).all()
    from sglang_omni_b200.models.ming_omni.audio_vae import StreamingVAEDecoder

    sv = StreamingVAEDecoder(vae, context=64)
    parts = [sv.push(z[0, :4]), sv.push(z[0, 4:7]), sv.push(z[0, 7:], last=True)]
    got = torch.cat(parts)
    assert got.shape == full.shape
    assert float((got - full).abs().max() / full.abs().max()) < 1e-3


def test_talker_prompt_layout():
    from sglang_omni_b200.models.common.tokenizer import SpecialsByteTokenizer
    from sglang_omni_b200.models.ming_omni.loader import TALKER_SPECIALS

    tok = SpecialsByteTokenizer(TALKER_SPECIALS, 1024, eos="<|endoftext|>")
    ids, rows = build_talker_prompt(tok, "hello there", n_speakers=1, n_prompt_latents=3, prompt_text="ref")
    text = tok.decode(ids, skip_special_tokens=False)
    assert "speaker_1:<|vision_start|><|vision_pad|><|vision_end|>" in text
    assert text.endswith("<|im_start|>assistant\n<audio><audioPatch><audioPatch><audioPatch>")
    assert ids[rows["spk"][0] - 1] == tok.convert_tokens_to_ids("<|vision_start|>")
    assert [ids[r] for r in rows["latent"]] == [tok.convert_tokens_to_ids("<audioPatch>")] * 3


def _run_generator(device, dtype, use_graphs):
    torch.manual_seed(0)
    t = MingTalker(tiny_cfg(dtype), device=device).random_init_(seed=4, std=0.05)
    gen = MingSpeechGenerator(t, max_streams=4, max_context=256, use_graphs=use_graphs)
    streams = []
    for i, n in enumerate((10, 23, 7)):
        e = (torch.randn(n, t.cfg.llm.hidden_size, generator=torch.Generator().manual_seed(i)) * 0.1).to(device)
        streams.append(gen.add_stream(f"s{i}", e, max_patches=5 + i, min_patches=100))
    gen.run(streams)
    return streams


def test_generator_cpu():
    streams = _run_generator("cpu", torch.float32, False)
    for i, s in enumerate(streams):
        assert s.done and s.patches == 5 + i
        lat = torch.stack(s.latents)
        assert lat.shape == (5 + i, 4, 16) and torch.isfinite(lat).all()


TALKER_TINY = {"talker": dict(dit_hidden=96, dit_depth=2, dit_heads=4, agg_hidden=72, agg_depth=2, agg_heads=4,
                              history_patch_size=8, latent_dim=16, spk_dim=24),
               "talker_llm": LLM_TINY,
               "vae": dict(hop=40, hidden=64, layers=1, heads=1, kv_heads=1, intermediate=128)}


def _speech_pipeline(device):
    from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
    from sglang_omni_b200.config import PipelineRunner, compile_pipeline
    from sglang_omni_b200.models.ming_omni.config import MingOmniSpeechPipelineConfig, ming_speech_stages
    from test_ming import TINY

    ov = {**TINY, **TALKER_TINY}
    st = ming_speech_stages(overrides=ov, device=device, max_batch=4, max_context=1024, max_streams=4)
    for s in st:
        if s.name == "talker":
            s.executor.args["max_patches"] = 6
    cfg = MingOmniSpeechPipelineConfig(model_path="random", stages=st)

    async def main():
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            client = Client(coord)
            reqs = [GenerateRequest(prompt=p, max_tokens=5, stream=False, output_modalities=["text", "audio"],
                                    sampling=SamplingParams(temperature=0.0, ignore_eos=True))
                    for p in ("Hello", "Say something")]
            return await asyncio.gather(*[_chunks(client, r) for r in reqs])

    return asyncio.run(main())


async def _chunks(client, req):
    return [ch async for ch in client.generate(req)]


def _check_speech(outs):
    for chunks in outs:
        audio = [c for c in chunks if c.audio_data is not None]
        assert len(audio) == 1 and audio[0].sample_rate == 16000
        # at most 6 patches x 4 latent frames x 4 decoder frames x 40 samples
        assert 0 < np.asarray(audio[0].audio_data).size <= 6 * 4 * 4 * 40
        assert any(c.text for c in chunks)


def test_ming_speech_pipeline_cpu_end_to_end():
    _check_speech(_speech_pipeline("cpu"))


# ----------------------------------------------------------------------------- GPU tier
@pytest.mark.gpu
def test_talker_modules_gpu_match_cpu():
    torch.manual_seed(0)
    cpu = MingTalker(tiny_cfg()).random_init_(seed=3, std=0.05)
    gpu = MingTalker(tiny_cfg(torch.bfloat16), device="cuda")
    with torch.no_grad():
        for (_, a), (_, b) in zip(cpu.named_parameters(), gpu.named_parameters()):
            b.copy_(a.to(b.dtype))
    c = cpu.cfg
    B = 3
    cond = torch.randn(B, c.llm.hidden_size)
    his = torch.randn(B, c.history_patch_size, c.latent_dim)
    x = torch.randn(B, c.patch_size, c.latent_dim)
    L = 1 + c.history_patch_size + c.patch_size
    ref = velocity_oracle(cpu, x, torch.full((B,), 0.3), cond, his)
    d = lambda t: t.cuda().bfloat16()  # noqa: E731
    v = gpu.dit_velocity(d(x), torch.full((B,), 0.3, device="cuda"), d(cond), d(his), RowLayout(B, L, "cuda"))
    assert float((v.float().cpu() - ref).norm() / ref.norm()) < 0.03
    ref_a = aggregate_oracle(cpu, x)
    a = gpu.aggregate(d(x), RowLayout(B, 1 + c.patch_size, "cuda"))
    assert float((a.float().cpu() - ref_a).norm() / ref_a.norm()) < 0.03


@pytest.mark.gpu
@pytest.mark.parametrize("graphs", [False, True])
def test_generator_gpu(graphs):
    streams = _run_generator("cuda", torch.bfloat16, graphs)
    for i, s in enumerate(streams):
        lat = torch.stack(s.latents)
        assert s.done and lat.shape == (5 + i, 4, 16) and torch.isfinite(lat).all()


@pytest.mark.gpu
def test_vae_decode_gpu_matches_cpu():
    cfg32 = AudioVAEConfig(hop=40, hidden=64, layers=2, heads=1, kv_heads=1, intermediate=128, latent_dim=16,
                           dtype=torch.float32)
    cfg16 = AudioVAEConfig(hop=40, hidden=64, layers=2, heads=1, kv_heads=1, intermediate=128, latent_dim=16)
    cpu = AudioVAEDecoder(cfg32).random_init_(seed=2, std=0.05)
    gpu = AudioVAEDecoder(cfg16, device="cuda")
    with torch.no_grad():
        for (_, a), (_, b) in zip(cpu.named_parameters(), gpu.named_parameters()):
            b.copy_(a.to(b.dtype))
    z = torch.randn(2, 9, 16)
    ref = cpu.decode(z)
    got = gpu.decode(z.cuda()).cpu()
    assert float((got - ref).norm() / ref.norm()) < 0.05


@pytest.mark.gpu
def test_ming_speech_pipeline_gpu_end_to_end():
    _check_speech(_speech_pipeline("cuda:0"))
