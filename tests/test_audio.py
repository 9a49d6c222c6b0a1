"""Audio tower and log-mel front-end against their oracles (HF module / torch.stft)."""
import numpy as np
import pytest
import torch

from sglang_omni_b200.models.qwen3_omni.audio_encoder import AudioEncoderConfig, Qwen3OmniAudioEncoder
from sglang_omni_b200.ops.mel import LogMel, mel_filters

hf = pytest.importorskip("transformers.models.qwen3_omni_moe.modeling_qwen3_omni_moe")
hfc = pytest.importorskip("transformers.models.qwen3_omni_moe.configuration_qwen3_omni_moe")


def tiny_hf():
    cfg = hfc.Qwen3OmniMoeAudioEncoderConfig(num_mel_bins=16, encoder_layers=2, encoder_attention_heads=4,
                                             encoder_ffn_dim=128, d_model=64, n_window=50, n_window_infer=400,
                                             downsample_hidden_size=8, output_dim=32, max_source_positions=200)
    cfg._attn_implementation = "eager"
    torch.manual_seed(0)
    m = hf.Qwen3OmniMoeAudioEncoder(cfg).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            p.copy_(torch.randn_like(p) * (0.2 if p.dim() > 1 else 0.05) + (1.0 if "norm" in n and "weight" in n else 0))
    return cfg, m


def test_audio_encoder_matches_hf_cpu():
    cfg, m = tiny_hf()
    ours = Qwen3OmniAudioEncoder(AudioEncoderConfig(num_mel_bins=16, encoder_layers=2, encoder_attention_heads=4,
                                                    encoder_ffn_dim=128, d_model=64, downsample_hidden_size=8,
                                                    output_dim=32, max_source_positions=200, dtype=torch.float32))
    ours.load_hf_state_dict(m.state_dict())
    # HF's eager / sdpa audio attention ignores cu_seqlens (only its flash-attention
    # path windows), so the oracle comparison uses one request that fits in a
    # single 52-token window (400 frames); windowing is checked separately below.
    mel = torch.randn(16, 400)
    with torch.no_grad():
        ref = m(mel, feature_lens=torch.tensor([400])).last_hidden_state
        out = ours([mel])[0]
    assert out.shape == ref.shape == (52, 32), (out.shape, ref.shape)
    assert (out - ref).abs().max() / ref.abs().max() < 1e-3


def test_audio_encoder_windows_are_block_diagonal():
    cfg, m = tiny_hf()
    ours = Qwen3OmniAudioEncoder(AudioEncoderConfig(num_mel_bins=16, encoder_layers=2, encoder_attention_heads=4,
                                                    encoder_ffn_dim=128, d_model=64, downsample_hidden_size=8,
                                                    output_dim=32, max_source_positions=200, dtype=torch.float32))
    ours.load_hf_state_dict(m.state_dict())
    a, b = torch.randn(16, 1000), torch.randn(16, 230)
    with torch.no_grad():
        both = ours([a, b])
        sa = ours([a])[0]
        sb = ours([b])[0]
        # the first window of `a` only sees itself: equals encoding its first 400 frames
        first = ours([a[:, :400]])[0]
    assert both[0].shape == (130, 32) and both[1].shape[0] == 2 * 13 + 4
    torch.testing.assert_close(both[0], sa, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(both[1], sb, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(sa[:52], first, atol=1e-5, rtol=1e-5)


def test_mel_filters_shape_and_norm():
    f = mel_filters(128)
    assert f.shape == (128, 201) and (f >= 0).all()
    assert np.all(f.sum(1) > 0)


@pytest.mark.gpu
def test_logmel_gpu_matches_stft():
    torch.manual_seed(0)
    audio = torch.randn(16000 * 3) * 0.1
    ref = LogMel(128, "cpu")(audio)
    out = LogMel(128, "cuda")(audio).cpu()
    assert out.shape == ref.shape == (128, 300)
    assert (out - ref).abs().max() < 0.05


@pytest.mark.gpu
def test_logmel_batch_matches_single():
    """One batched call over waveforms of different lengths and loudness equals the per-waveform
    oracle (each waveform keeps its own bf16 range scales)."""
    torch.manual_seed(1)
    audios = [torch.randn(16000 * 2) * 0.1, torch.randn(12345) * 3.0, torch.randn(4000) * 1e-3,
              torch.randn(16000 * 2) * 2.0]   # equal lengths are framed together, scales stay per waveform
    outs = LogMel(128, "cuda").batch(audios)
    cpu = LogMel(128, "cpu")
    for a, o in zip(audios, outs):
        ref = cpu(a)
        assert o.shape == ref.shape
        assert (o.cpu() - ref).abs().max() < 0.05


@pytest.mark.gpu
def test_audio_encoder_gpu_matches_cpu():
    cfg = AudioEncoderConfig(num_mel_bins=128, encoder_layers=2, encoder_attention_heads=4, encoder_ffn_dim=512,
                             d_model=256, downsample_hidden_size=64, output_dim=128)
    cpu = Qwen3OmniAudioEncoder(AudioEncoderConfig(**{**cfg.__dict__, "dtype": torch.float32})).random_init_(
        seed=1, std=0.05)
    gpu = Qwen3OmniAudioEncoder(cfg, device="cuda")
    with torch.no_grad():
        for (n, a), (_, b) in zip(cpu.named_parameters(), gpu.named_parameters()):
            b.copy_(a.to(b.dtype))
    mels = [torch.randn(128, 1000) * 0.5, torch.randn(128, 370) * 0.5]
    ref = torch.cat(cpu(mels), 0)
    out = torch.cat(gpu([m.cuda() for m in mels]), 0).float().cpu()
    assert out.shape == ref.shape
    assert (out - ref).abs().max() / ref.abs().max() < 0.05
