"""Stateful streaming S2-Pro DAC decoding: chunks that run only their new code frames,
with the window transformer's keys / values and every convolution's history kept per
stream, concatenate to the full-sequence ``DACDecoder.decode`` of the same frames (the
oracle, itself checked against a plain-PyTorch restatement of the reference decoder)."""
import numpy as np
import pytest
import torch

from sglang_omni_b200.models.fishaudio_s2_pro.codec import DACConfig, DACDecoder, random_dac_state_dict
from sglang_omni_b200.models.fishaudio_s2_pro.codec_stateful import StatefulStreamingDAC, dac_conv_history

DAC_TINY = dict(latent_dim=64, decoder_dim=128, tf_layers=2, tf_heads=1, tf_head_dim=64, tf_inter=128,
                tf_window=8, encoder_dim=8, encoder_transformer_layers=(0, 0, 0, 1), n_codebooks=3,
                codebook_size=32, semantic_codebook_size=64)


def _codes(n_streams, T, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.stack([torch.randint(0, 64, (n_streams, T), generator=g)]
                       + [torch.randint(0, 32, (n_streams, T), generator=g) for _ in range(3)], 1)


def _feed(sc, names, codes, step_frames):
    out = {s: [] for s in names}
    for t in range(0, codes.shape[-1], step_frames):
        for i, s in enumerate(names):
            sc.add_codes(s, codes[i, :, t:t + step_frames].T)
        for r, w in sc.decode_ready(list(names)).items():
            out[r].append(np.asarray(w.cpu() if torch.is_tensor(w) else w))
    for r, w in sc.decode_ready(list(names), final=True).items():
        out[r].append(np.asarray(w.cpu() if torch.is_tensor(w) else w))
    return {s: np.concatenate(v) for s, v in out.items()}


def test_dac_history_sizes():
    cfg = DACConfig(**DAC_TINY, dtype=torch.float32)
    dec = DACDecoder(cfg).load_state_dict_dac(random_dac_state_dict(cfg, seed=1, std=0.05))
    hist = dac_conv_history(dec)
    assert len(hist) == 2 + 1 + 4 * 4 + 1 and hist[-1] == (6, 8)


@pytest.mark.parametrize("first_chunk,chunk,step_frames", [(5, 20, 3), (2, 3, 1)])
def test_dac_stateful_chunks_equal_full_decode(first_chunk, chunk, step_frames):
    cfg = DACConfig(**DAC_TINY, dtype=torch.float32)
    dec = DACDecoder(cfg).load_state_dict_dac(random_dac_state_dict(cfg, seed=1, std=0.05))
    T = 47
    codes = _codes(3, T, 5)
    sc = StatefulStreamingDAC(dec, chunk=chunk, first_chunk=first_chunk, max_streams=4, max_frames=256)
    got = _feed(sc, ["a", "b", "c"], codes, step_frames)
    ref = dec.decode(codes)
    for i, s in enumerate("abc"):
        assert got[s].shape == (T * cfg.hop,)
        np.testing.assert_allclose(got[s], ref[i].numpy(), atol=1e-5, rtol=1e-4)


def test_dac_stateful_ring_wrap_and_slot_reuse():
    cfg = DACConfig(**DAC_TINY, dtype=torch.float32)
    dec = DACDecoder(cfg).load_state_dict_dac(random_dac_state_dict(cfg, seed=3, std=0.05))
    sc = StatefulStreamingDAC(dec, chunk=7, first_chunk=3, max_streams=1, max_frames=512)
    assert sc.state.kv.ring * 64 < 140
    a, b = _codes(1, 140, 7)[0], _codes(1, 20, 8)[0]
    got_a = _feed(sc, ["a"], a[None], 4)["a"]
    sc.close("a")                      # "b" takes the same slot and must not see a's state
    got_b = _feed(sc, ["b"], b[None], 4)["b"]
    np.testing.assert_allclose(got_a, dec.decode(a[None])[0].numpy(), atol=1e-5, rtol=1e-4)
    np.testing.assert_allclose(got_b, dec.decode(b[None])[0].numpy(), atol=1e-5, rtol=1e-4)


@pytest.mark.gpu
def test_dac_stateful_gpu_matches_cpu_oracle_and_graphs():
    cpu_cfg = DACConfig(**DAC_TINY, dtype=torch.float32)
    sd = random_dac_state_dict(cpu_cfg, seed=4, std=0.05)
    cpu = DACDecoder(cpu_cfg).load_state_dict_dac(sd)
    gpu = DACDecoder(DACConfig(**DAC_TINY), "cuda").load_state_dict_dac(sd)
    T = 83
    codes = _codes(5, T, 9)
    ref = cpu.decode(codes).numpy()
    for use_graphs in (False, True):
        sc = StatefulStreamingDAC(gpu, chunk=20, first_chunk=5, max_streams=8, max_frames=256,
                                  use_graphs=use_graphs)
        sc.capture_graphs()
        got = _feed(sc, [f"s{i}" for i in range(5)], codes.cuda(), 6)
        for i in range(5):
            g = got[f"s{i}"]
            assert g.shape == ref[i].shape
            rel = np.linalg.norm(g - ref[i]) / max(np.linalg.norm(ref[i]), 1e-6)
            assert rel < 0.05, (use_graphs, i, rel)
