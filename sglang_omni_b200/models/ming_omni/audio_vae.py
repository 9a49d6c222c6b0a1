"""Ming-Omni AudioVAE decoder: talker latents -> waveform.

latents [B, T, Z] -> linear to the decoder width -> linear-interpolation
upsampling by ``patch_size`` along time -> causal Qwen2-style transformer
(the shared ``DecoderLM`` layers on the paged kernels, one prefill per call)
-> ISTFT head: a linear layer predicts log-magnitude and phase of n_fft/2 + 1
bins per frame, the inverse real DFT with the synthesis window folded in runs
as ONE GEMM ([frames, 2 (n_fft/2 + 1)] x [2 (n_fft/2 + 1), n_fft]) on the
tcgen05 kernel, then overlap-add with hop ``hop`` (window = n_fft = 4 hop, so
every output hop sums four frame quarters), normalised by the overlap-added
squared window and trimmed by (n_fft - hop) / 2 on both sides ("same" padding).

Streaming (``StreamingVAEDecoder``) re-decodes a bounded window of the latest
latents and emits only the samples that no later latent can change.

Reference counterparts: AudioVAE.decode / Decoder.low_level_reconstruct /
StreamingLinearUpsample (sglang_omni/models/ming_omni/talker/audio_vae/
modeling_audio_vae.py:12-99, vae_modules.py:9-235) and ISTFT / ISTFTHead
(talker/audio_vae/istft.py:5-219).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

from ... import ops
from ...engines.ar.kv_pool import KVPool
from ...utils.hostdev import h2d
from ..decoder import DecoderConfig, DecoderLM, ForwardBatch


@dataclass
class AudioVAEConfig:
    sample_rate: int = 16000
    latent_dim: int = 64
    hop: int = 320            # output samples per decoder frame (the decoder's output_dim)
    patch_size: int = 4       # decoder frames per latent
    hidden: int = 896
    layers: int = 12
    heads: int = 14
    kv_heads: int = 2
    intermediate: int = 4864
    rope_theta: float = 1e6
    dtype: torch.dtype = torch.bfloat16

    @property
    def n_fft(self) -> int:
        return 4 * self.hop

    def decoder_config(self) -> DecoderConfig:
        return DecoderConfig(vocab_size=16, hidden_size=self.hidden, num_layers=self.layers, num_heads=self.heads,
                             num_kv_heads=self.kv_heads, head_dim=self.hidden // self.heads,
                             intermediate_size=self.intermediate, rope_theta=self.rope_theta, qk_norm=False,
                             attention_bias=True, max_position=65536, dtype=self.dtype, name="ming_vae_decoder")

    @classmethod
    def from_dict(cls, raw: dict) -> "AudioVAEConfig":
        dec = (raw.get("dec_kwargs") or {})
        bb = dec.get("backbone") or {}
        heads = bb.get("num_attention_heads", 14)
        return cls(sample_rate=raw.get("sample_rate", 16000), latent_dim=dec.get("latent_dim", 64),
                   hop=dec.get("output_dim", 320), patch_size=raw.get("patch_size", 4),
                   hidden=bb.get("hidden_size", 896), layers=bb.get("num_hidden_layers", 12), heads=heads,
                   kv_heads=bb.get("num_key_value_heads", heads), intermediate=bb.get("intermediate_size", 4864),
                   rope_theta=bb.get("rope_theta", 1e6))


def irfft_basis(n_fft: int, window: torch.Tensor) -> torch.Tensor:
    """[n_fft, 2 * (n_fft/2 + 1)]: columns (Re X_k, Im X_k) -> windowed time sample n of the
    inverse real DFT, x[n] = (1/N) sum_k c_k (Re X_k cos(2 pi k n / N) - Im X_k sin(2 pi k n / N)),
    c_0 = c_{N/2} = 1, otherwise 2 (the imaginary parts of bins 0 and N/2 drop out)."""
    N = n_fft
    K = N // 2 + 1
    n = torch.arange(N, dtype=torch.float64)[:, None]
    k = torch.arange(K, dtype=torch.float64)[None, :]
    c = torch.full((1, K), 2.0, dtype=torch.float64)
    c[0, 0] = 1.0
    c[0, -1] = 1.0
    ang = 2 * math.pi * n * k / N
    re = c * torch.cos(ang) / N
    im = -c * torch.sin(ang) / N
    im[:, 0] = 0.0
    im[:, -1] = 0.0
    return (torch.cat([re, im], 1) * window.double()[:, None]).float()


def overlap_add4(frames: torch.Tensor, hop: int) -> torch.Tensor:
    """frames [B, T, 4 hop] (window = 4 hops) -> [B, (T + 3) hop] overlap-added signal."""
    B, T, W = frames.shape
    q = frames.view(B, T, 4, hop)
    out = frames.new_zeros(B, T + 3, hop)
    for j in range(4):
        out[:, j:j + T] += q[:, :, j]
    return out.reshape(B, (T + 3) * hop)


class AudioVAEDecoder(nn.Module):
    def __init__(self, cfg: AudioVAEConfig = AudioVAEConfig(), device="cpu"):
        super().__init__()
        self.cfg = cfg
        dt = cfg.dtype
        P = lambda *s: nn.Parameter(torch.empty(*s, dtype=dt, device=device), requires_grad=False)  # noqa: E731
        self.fc1, self.fc1_b = P(cfg.hidden, cfg.latent_dim), P(cfg.hidden)
        self.lm = DecoderLM(cfg.decoder_config(), device=device)
        K = cfg.n_fft // 2 + 1
        self.head, self.head_b = P(2 * K, cfg.hidden), P(2 * K)
        win = torch.hann_window(cfg.n_fft, periodic=True, dtype=torch.float64)
        self.register_buffer("window", win.float().to(device), persistent=False)
        # the GEMM wants K % 8 == 0: zero columns pad the (Re, Im) spectrum axis
        self.k_pad = (2 * K + 7) // 8 * 8
        basis = torch.zeros(cfg.n_fft, self.k_pad, dtype=torch.float32)
        basis[:, :2 * K] = irfft_basis(cfg.n_fft, win)
        self.register_buffer("basis", basis.to(dt).to(device), persistent=False)

    @property
    def device(self):
        return self.fc1.device

    def random_init_(self, seed: int = 0, std: float = 0.02):
        self.lm.random_init_(seed=seed, std=std)
        g = torch.Generator().manual_seed(seed + 5)
        for p in (self.fc1, self.fc1_b, self.head, self.head_b):
            p.copy_((torch.randn(p.shape, generator=g) * std).to(p.dtype))
        return self

    def load_state_dict_ref(self, sd: dict[str, torch.Tensor], prefix: str = "decoder."):
        """From the reference layout (``decoder.fc1``, ``decoder.decoder.*`` Qwen2,
        ``decoder.head.out``); the layer norms of the backbone are its own."""
        from ..weight_loader import load_decoder_from_hf

        self.fc1.copy_(sd[prefix + "fc1.weight"])
        self.fc1_b.copy_(sd[prefix + "fc1.bias"])
        load_decoder_from_hf(self.lm, sd, prefix + "decoder.", lm_head_key=None, embed_key="__none__")
        self.head.copy_(sd[prefix + "head.out.weight"])
        self.head_b.copy_(sd[prefix + "head.out.bias"])

    # ------------------------------------------------------------------ pieces
    def upsample(self, x: torch.Tensor) -> torch.Tensor:
        """Linear interpolation by patch_size along time (half-pixel centres, edges clamped)."""
        if self.cfg.patch_size == 1:
            return x
        y = F.interpolate(x.float().transpose(1, 2), scale_factor=self.cfg.patch_size, mode="linear",
                          align_corners=False)
        return y.transpose(1, 2).to(x.dtype).contiguous()

    def backbone(self, h: torch.Tensor) -> torch.Tensor:
        """Causal transformer over every sequence of h [B, L, hidden] (one paged prefill)."""
        B, L, H = h.shape
        lm = self.lm
        dev = h.device
        pages_per = KVPool.pages_for(L)
        pool = KVPool(lm.cfg.num_layers, lm.cfg.num_kv_heads, lm.cfg.head_dim, B * pages_per + 1, dev, lm.cfg.dtype)
        lm.ensure_workspaces(B * L, B, pages_per * 64)
        pages = np.arange(1, B * pages_per + 1, dtype=np.int32).reshape(B, pages_per)
        t = np.arange(L)
        slots = (pages[:, t // 64] * 64 + t % 64).reshape(-1).astype(np.int32)
        pos = np.tile(np.arange(L, dtype=np.int32), B)
        cu = np.arange(0, (B + 1) * L, L, dtype=np.int32)
        req, tok0 = ops.prefill_tiles([L] * B, lm.cfg.num_heads // lm.cfg.num_kv_heads)
        d = lambda a: h2d(a, dev)  # noqa: E731
        fb = ForwardBatch(is_decode=False, positions=d(np.stack([pos] * 3)), slot_mapping=d(slots),
                          kv_lens=h2d([L] * B, dev, torch.int32), block_table=d(pages), cu_q=d(cu),
                          input_embeds=h.reshape(B * L, H).to(lm.cfg.dtype),
                          tile_req=h2d(req, dev, torch.int32), tile_tok0=h2d(tok0, dev, torch.int32))
        return lm(fb, pool.kv).view(B, L, H)

    def istft_head(self, h: torch.Tensor) -> torch.Tensor:
        """[B, L, hidden] -> [B, L * hop] waveform."""
        cfg = self.cfg
        B, L, _ = h.shape
        K = cfg.n_fft // 2 + 1
        pred = ops.linear(h.reshape(B * L, -1), self.head, bias=self.head_b, out_dtype=torch.float32)
        mag = torch.exp(pred[:, :K]).clamp(max=1e2)
        ph = pred[:, K:]
        spec = torch.zeros(B * L, self.k_pad, dtype=cfg.dtype, device=h.device)   # [B L, 2K + pad] (Re, Im)
        spec[:, :K] = mag * torch.cos(ph)
        spec[:, K:2 * K] = mag * torch.sin(ph)
        frames = ops.linear(spec, self.basis, out_dtype=torch.float32).view(B, L, cfg.n_fft)
        y = overlap_add4(frames, cfg.hop)
        env = overlap_add4(self.window.square().expand(1, L, cfg.n_fft).contiguous(), cfg.hop)
        pad = (cfg.n_fft - cfg.hop) // 2
        y = y[:, pad:y.shape[1] - pad]
        env = env[:, pad:env.shape[1] - pad]
        return y / env.clamp_min(1e-11)

    @torch.no_grad()
    def decode(self, latents: torch.Tensor) -> torch.Tensor:
        """latents [B, T, Z] -> waveform [B, T * patch_size * hop] (float32)."""
        x = ops.linear(latents.to(self.cfg.dtype).reshape(-1, self.cfg.latent_dim), self.fc1, bias=self.fc1_b)
        x = self.upsample(x.view(latents.shape[0], latents.shape[1], -1))
        h = self.backbone(x)
        return self.istft_head(h)


class StreamingVAEDecoder:
    """Chunked decoding of a growing latent sequence: each call decodes the last
    ``context`` latents plus the new ones and returns only the samples that are
    final (one latent of look-ahead is held back for the interpolation and the
    overlap-add tail until ``last``)."""

    def __init__(self, vae: AudioVAEDecoder, context: int = 64):
        self.vae = vae
        self.context = context
        self.latents: list[torch.Tensor] = []
        self.emitted = 0          # samples already returned

    def push(self, new: torch.Tensor, last: bool = False) -> torch.Tensor:
        """new: [n, Z] latents; returns the next samples (float32, possibly empty)."""
        if new is not None and new.numel():
            self.latents.append(new.float().cpu())
        if not self.latents:
            return torch.zeros(0)
        allz = torch.cat(self.latents, 0)
        n = allz.shape[0]
        spl = self.vae.cfg.patch_size * self.vae.cfg.hop   # samples per latent
        start = max(0, n - self.context - 1)
        wav = self.vae.decode(allz[start:].unsqueeze(0).to(self.vae.device))[0].cpu()
        final_end = n * spl if last else max(0, (n - 1) * spl - self.vae.cfg.n_fft)
        lo = self.emitted - start * spl
        if final_end <= self.emitted or lo < 0:
            return torch.zeros(0)
        out = wav[lo:final_end - start * spl]
        self.emitted = final_end
        return out
