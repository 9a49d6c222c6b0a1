"""Code2Wav (vocoder) against the HF transformers implementation on CPU, and
the GPU kernels path against the CPU path."""
import pytest
import torch

from sglang_omni_b200.models.qwen3_omni.code2wav import Code2Wav, Code2WavConfig, StreamingCode2Wav

hf = pytest.importorskip("transformers.models.qwen3_omni_moe.modeling_qwen3_omni_moe")
hfc = pytest.importorskip("transformers.models.qwen3_omni_moe.configuration_qwen3_omni_moe")


def tiny_hf():
    cfg = hfc.Qwen3OmniMoeCode2WavConfig(codebook_size=32, hidden_size=64, num_attention_heads=4,
                                         num_key_value_heads=4, sliding_window=8, intermediate_size=128,
                                         num_hidden_layers=2, num_quantizers=4, upsample_rates=(2, 3),
                                         upsampling_ratios=(2,), decoder_dim=32)
    torch.manual_seed(0)
    m = hf.Qwen3OmniMoeCode2Wav(cfg).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if "alpha" in n or "beta" in n:
                p.copy_(torch.randn_like(p) * 0.3)
            elif "scale" in n or "gamma" in n:
                p.copy_(torch.rand_like(p) * 0.5 + 0.1)
            elif p.dim() > 1:
                p.copy_(torch.randn_like(p) * 0.15)
            else:
                p.copy_(torch.randn_like(p) * 0.05 + (1.0 if "norm" in n and "weight" in n else 0.0))
    return cfg, m


def ours_from(cfg, m, dtype=torch.float32, device="cpu"):
    c = Code2WavConfig(codebook_size=cfg.codebook_size, hidden_size=cfg.hidden_size,
                       num_heads=cfg.num_attention_heads, num_kv_heads=cfg.num_key_value_heads,
                       sliding_window=cfg.sliding_window, intermediate_size=cfg.intermediate_size,
                       num_layers=cfg.num_hidden_layers, num_quantizers=cfg.num_quantizers,
                       upsample_rates=tuple(cfg.upsample_rates), upsampling_ratios=tuple(cfg.upsampling_ratios),
                       decoder_dim=cfg.decoder_dim, rms_norm_eps=cfg.rms_norm_eps, dtype=dtype,
                       rope_theta=float((cfg.rope_parameters or {}).get("rope_theta", 10000.0)))
    ours = Code2Wav(c, device=device)
    ours.load_hf_state_dict({k: v.to(device) for k, v in m.state_dict().items()})
    return ours


def test_code2wav_matches_hf_cpu():
    cfg, m = tiny_hf()
    ours = ours_from(cfg, m)
    codes = torch.randint(0, cfg.codebook_size, (2, cfg.num_quantizers, 11))
    with torch.no_grad():
        ref = m(codes).squeeze(1)
        out = ours(codes)
    assert out.shape == ref.shape
    err = (out - ref).abs().max() / ref.abs().max().clamp_min(1e-6)
    assert err < 2e-3, float(err)


def test_streaming_matches_windowed_decode():
    cfg, m = tiny_hf()
    ours = ours_from(cfg, m)
    st = StreamingCode2Wav(ours, chunk=3, left_context=4)
    codes = torch.randint(0, cfg.codebook_size, (cfg.num_quantizers, 13))
    outs = []
    for t in range(13):
        st.add_codes("r", codes[:, t])
        outs += [w for w in st.decode_ready(["r"]).values()]
    outs += [w for w in st.decode_ready(["r"], final=True).values()]
    # chunks at frames 3, 6, 9, 12 and the final partial one
    assert len(outs) == 5 and all(o.numel() > 0 for o in outs)
    # the first chunk has no left context: it equals the plain decode of the first frames
    first = ours(codes[None, :, :3])[0]
    torch.testing.assert_close(outs[0], first, atol=1e-5, rtol=1e-5)
    # a later chunk equals the windowed decode (context 4) minus the context samples, as in HF chunked_decode
    up = ours.cfg.total_upsample
    win = ours(codes[None, :, 2:9])[0]
    torch.testing.assert_close(outs[2], win[4 * up:], atol=1e-5, rtol=1e-5)


@pytest.mark.gpu
def test_code2wav_gpu_matches_cpu():
    cfg = Code2WavConfig(codebook_size=64, hidden_size=256, num_heads=4, num_kv_heads=4, sliding_window=16,
                         intermediate_size=512, num_layers=2, num_quantizers=4, upsample_rates=(4, 2),
                         upsampling_ratios=(2,), decoder_dim=256)
    cpu = Code2Wav(Code2WavConfig(**{**cfg.__dict__, "dtype": torch.float32})).random_init_(seed=3, std=0.02)
    gpu = Code2Wav(cfg, device="cuda")
    with torch.no_grad():
        for (n, a), (_, b) in zip(cpu.named_parameters(), gpu.named_parameters()):
            b.copy_(a.to(b.dtype))
        for n, p in cpu.named_parameters():
            if n.endswith(("snake_a", "snake_b", "a1", "b1", "a2", "b2")):
                p.copy_(torch.randn_like(p) * 0.1)
        for (n, a), (_, b) in zip(cpu.named_parameters(), gpu.named_parameters()):
            b.copy_(a.to(b.dtype))
    codes = torch.randint(0, 64, (3, 4, 20))
    with torch.no_grad():
        ref = cpu(codes)
        out = gpu(codes.cuda()).cpu()
    # bf16 kernels vs the fp32 oracle: relative L2 error of the waveform
    assert float((out - ref).norm() / ref.norm().clamp_min(1e-6)) < 0.05


@pytest.mark.gpu
def test_code2wav_graphs_match_eager():
    """Captured (batch bucket, window) graphs give the eager forward's waveform, padded
    batches and uncaptured windows included, and the streaming decoder's host output is
    the same through graphs as without."""
    from sglang_omni_b200.models.qwen3_omni.code2wav import Code2WavGraphs, chunk_windows

    cfg = Code2WavConfig(codebook_size=64, hidden_size=256, num_heads=4, num_kv_heads=4, sliding_window=16,
                         intermediate_size=512, num_layers=2, num_quantizers=4, upsample_rates=(4, 2),
                         upsampling_ratios=(2,), decoder_dim=256)
    m = Code2Wav(cfg, device="cuda").random_init_(seed=4, std=0.05)
    g = Code2WavGraphs(m, max_batch=8)
    wins = chunk_windows(3, 4, 2)
    g.capture_windows(wins)
    gen = torch.Generator().manual_seed(1)
    with torch.no_grad():
        for B in (1, 3, 8):
            for W in wins + [5]:          # 5 is not captured: eager
                codes = torch.randint(0, 64, (B, 4, W), generator=gen).cuda()
                ref = m(codes)
                got = g(codes).clone()
                torch.testing.assert_close(got, ref, atol=2e-3, rtol=1e-3)
    a = StreamingCode2Wav(m, chunk=3, left_context=4, first_chunk=2, graphs=g)
    b = StreamingCode2Wav(m, chunk=3, left_context=4, first_chunk=2)
    codes = torch.randint(0, 64, (5, 4, 14), generator=gen)
    for t in range(14):
        for s in range(5):
            a.add_codes(f"s{s}", codes[s, :, t])
            b.add_codes(f"s{s}", codes[s, :, t])
        ra = a.decode_ready([f"s{s}" for s in range(5)], to_host=True)
        rb = b.decode_ready([f"s{s}" for s in range(5)])
        assert ra.keys() == rb.keys()
        for k in ra:
            torch.testing.assert_close(torch.from_numpy(ra[k]), rb[k].float().cpu(), atol=2e-3, rtol=1e-3)
