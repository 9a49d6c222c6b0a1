"""Stateful streaming Code2Wav: chunks that run only their new frames, with the
transformer's keys / values and every convolution's history kept per stream,
concatenate to the full-sequence forward of the same frames (the oracle:
``Code2Wav.forward`` on CPU, itself checked against transformers' module)."""
import numpy as np
import pytest
import torch

from sglang_omni_b200.models.qwen3_omni.code2wav import Code2Wav, Code2WavConfig
from sglang_omni_b200.models.qwen3_omni.code2wav_stateful import (StatefulStreamingCode2Wav, conv_history,
                                                                  first_chunk_samples)


def tiny(dtype=torch.float32, device="cpu", seed=3, hidden=64):
    """head_dim = hidden / 4 (the GPU kernels take head dims 32, 64, 96 and 128)."""
    cfg = Code2WavConfig(codebook_size=32, hidden_size=hidden, num_heads=4, num_kv_heads=4, sliding_window=8,
                         intermediate_size=2 * hidden, num_layers=2, num_quantizers=4, upsample_rates=(2, 3),
                         upsampling_ratios=(2,), decoder_dim=32, dtype=dtype)
    m = Code2Wav(cfg, device=device).random_init_(seed=seed, std=0.05)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if n.endswith(("snake_a", "snake_b", "a1", "b1", "a2", "b2")):
                p.copy_((torch.randn(p.shape, generator=g) * 0.3).to(p.dtype))
            elif n.endswith(("attn_scale", "mlp_scale")):
                p.copy_((torch.rand(p.shape, generator=g) * 0.5 + 0.1).to(p.dtype))
    return m


def _feed(sc, streams, codes, step_frames):
    """Feeds every stream's frames in interleaved steps; returns {stream: concatenated wave}."""
    out = {s: [] for s in streams}
    T = codes.shape[-1]
    for t in range(0, T, step_frames):
        for i, s in enumerate(streams):
            sc.add_codes(s, codes[i, :, t:t + step_frames].T)
        for r, w in sc.decode_ready(list(streams)).items():
            out[r].append(np.asarray(w.cpu() if torch.is_tensor(w) else w))
    for r, w in sc.decode_ready(list(streams), final=True).items():
        out[r].append(np.asarray(w.cpu() if torch.is_tensor(w) else w))
    return {s: np.concatenate(v) for s, v in out.items()}


def test_history_sizes():
    m = tiny()
    hist = conv_history(m)
    # two upsample dwconvs + conv_in + 2 blocks x (tconv + 3 dilated units) + conv_out
    assert len(hist) == 1 + 1 + 2 * 4 + 1
    assert [n for n, _ in hist[3:6]] == [6, 18, 54]


@pytest.mark.parametrize("first_chunk,chunk,step_frames", [(2, 3, 1), (3, 3, 2), (1, 4, 5)])
def test_stateful_chunks_equal_full_sequence(first_chunk, chunk, step_frames):
    m = tiny()
    T = 23
    codes = torch.randint(0, 32, (3, 4, T), generator=torch.Generator().manual_seed(5))
    sc = StatefulStreamingCode2Wav(m, chunk=chunk, first_chunk=first_chunk, max_streams=4, max_frames=256)
    got = _feed(sc, ["a", "b", "c"], codes, step_frames)
    with torch.no_grad():
        ref = m(codes)
    assert ref.shape[1] == first_chunk_samples(m, T)
    for i, s in enumerate("abc"):
        assert got[s].shape == (ref.shape[1],), (got[s].shape, ref.shape)
        np.testing.assert_allclose(got[s], ref[i].numpy(), atol=1e-6, rtol=1e-5)


def test_stateful_long_stream_ring_and_slot_reuse():
    """Frames past several 64-key pages (the KV ring wraps), streams starting while others run,
    and a closed stream's slot reused by a new stream that must not see its state."""
    m = tiny(seed=7)
    sc = StatefulStreamingCode2Wav(m, chunk=5, first_chunk=2, max_streams=2, max_frames=512)
    g = torch.Generator().manual_seed(9)
    a = torch.randint(0, 32, (4, 300), generator=g)     # 300 keys: the 3-page (192-key) ring wraps
    b = torch.randint(0, 32, (4, 40), generator=g)
    c = torch.randint(0, 32, (4, 30), generator=g)
    outs = {"a": [], "b": [], "c": []}
    assert sc.state.kv.ring * 64 < 300
    for t in range(300):
        sc.add_codes("a", a[:, t])
        if t < 40:
            sc.add_codes("b", b[:, t])
        if t >= 60 and t - 60 < 30:
            sc.add_codes("c", c[:, t - 60])
        live = [r for r in ("a", "b", "c") if r in sc.streams]
        fins = {"b"} if t == 39 else ({"c"} if t == 89 else set())
        for r, w in sc.decode_ready(live, finals=fins).items():
            outs[r].append(w.numpy())
        if t == 39:
            sc.close("b")      # its slot goes to "c"
        if t == 89:
            sc.close("c")
    for r, w in sc.decode_ready(["a"], final=True).items():
        outs[r].append(w.numpy())
    with torch.no_grad():
        for name, codes in (("a", a), ("b", b), ("c", c)):
            ref = m(codes[None])[0].numpy()
            got = np.concatenate(outs[name])
            assert got.shape == ref.shape, name
            np.testing.assert_allclose(got, ref, atol=1e-6, rtol=1e-5, err_msg=name)


def test_stateful_capacity_errors():
    m = tiny()
    sc = StatefulStreamingCode2Wav(m, chunk=2, max_streams=1, max_frames=64)
    sc.add_codes("a", torch.zeros(4, dtype=torch.long))
    with pytest.raises(RuntimeError, match="open streams"):
        sc.add_codes("b", torch.zeros(4, dtype=torch.long))
    sc.add_codes("a", torch.zeros(70, 4, dtype=torch.long))
    with pytest.raises(ValueError, match="max_frames"):
        sc.decode_ready(["a"], final=True)


@pytest.mark.gpu
def test_stateful_gpu_matches_cpu_oracle_and_graphs():
    """bf16 kernels (paged sliding-window attention over the KV ring, RoPE + KV store, conv
    GEMMs) against the fp32 full-sequence oracle, eager and through captured graphs."""
    cpu = tiny(seed=11, hidden=256)     # head_dim 64, as in the released model
    cfg = Code2WavConfig(**{**cpu.cfg.__dict__, "dtype": torch.bfloat16})
    gpu = Code2Wav(cfg, device="cuda")
    with torch.no_grad():
        for (_, a), (_, b) in zip(cpu.named_parameters(), gpu.named_parameters()):
            b.copy_(a.to(b.dtype))
    T = 97
    codes = torch.randint(0, 32, (5, 4, T), generator=torch.Generator().manual_seed(13))
    with torch.no_grad():
        ref = cpu(codes).numpy()
    for use_graphs in (False, True):
        sc = StatefulStreamingCode2Wav(gpu, chunk=10, first_chunk=2, max_streams=8, max_frames=256,
                                       use_graphs=use_graphs)
        sc.capture_graphs()
        got = _feed(sc, [f"s{i}" for i in range(5)], codes.cuda(), 3)
        for i in range(5):
            g = got[f"s{i}"]
            assert g.shape == ref[i].shape
            rel = np.linalg.norm(g - ref[i]) / max(np.linalg.norm(ref[i]), 1e-6)
            assert rel < 0.05, (use_graphs, i, rel)
