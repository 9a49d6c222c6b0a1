"""Qwen3-Omni audio tower on the sm_100a ops.

log-mel [128, T] per request -> 200-frame chunks -> 3 x (Conv2d 3x3 s2 p1 +
GELU), channels-last implicit im2col + tcgen05 GEMM with the bias/GELU fused
-> Linear(480*16 -> d) -> + sinusoid positions (restarting every chunk) ->
32 x [LN, MHA (varlen, block-diagonal over 50-token windows), LN, GELU FFN]
-> LN -> proj1 -> GELU -> proj2 (-> thinker hidden).  All chunks of all
requests of a batch go through one set of launches.

Architecture and window arithmetic follow transformers
Qwen3OmniMoeAudioEncoder (used by
sglang_omni/models/qwen3_omni/components/audio_encoder.py:37-89): chunk
2*n_window frames, window n_window_infer / (2*n_window) chunks.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
from torch import nn

from ... import ops
from ...ops import audio as A


@dataclass
class AudioEncoderConfig:
    num_mel_bins: int = 128
    encoder_layers: int = 32
    encoder_attention_heads: int = 20
    encoder_ffn_dim: int = 5120
    d_model: int = 1280
    n_window: int = 50
    n_window_infer: int = 400
    downsample_hidden_size: int = 480
    output_dim: int = 2048
    max_source_positions: int = 1500
    dtype: torch.dtype = torch.bfloat16

    @property
    def freq_after_cnn(self):
        return (((self.num_mel_bins + 1) // 2 + 1) // 2 + 1) // 2


def cnn_out_len(n: int) -> int:
    """Tokens produced by the 3 stride-2 convs for a chunk of n frames."""
    for _ in range(3):
        n = (n - 1) // 2 + 1
    return n


def sinusoids(length: int, channels: int, max_timescale: float = 10000.0) -> torch.Tensor:
    inc = np.log(max_timescale) / (channels // 2 - 1)
    inv = torch.exp(-inc * torch.arange(channels // 2).float())
    t = torch.arange(length)[:, None].float() * inv[None, :]
    return torch.cat([torch.sin(t), torch.cos(t)], 1)


class Qwen3OmniAudioEncoder(nn.Module):
    def __init__(self, cfg: AudioEncoderConfig | None = None, device="cpu"):
        super().__init__()
        cfg = cfg or AudioEncoderConfig()
        self.cfg = cfg
        d, C, dt = cfg.d_model, cfg.downsample_hidden_size, cfg.dtype
        P = lambda *s: nn.Parameter(torch.empty(*s, dtype=dt, device=device), requires_grad=False)  # noqa: E731
        self.conv1_w, self.conv1_b = P(C, 16), P(C)          # 9 taps padded to 16 (TMA row alignment)
        self.conv2_w, self.conv2_b = P(C, 9 * C), P(C)
        self.conv3_w, self.conv3_b = P(C, 9 * C), P(C)
        self.conv_out_w = P(d, C * cfg.freq_after_cnn)
        self.layers = nn.ModuleList()
        for _ in range(cfg.encoder_layers):
            L = nn.Module()
            L.ln1_w, L.ln1_b = P(d), P(d)
            L.qkv_w, L.qkv_b = P(3 * d, d), P(3 * d)
            L.o_w, L.o_b = P(d, d), P(d)
            L.ln2_w, L.ln2_b = P(d), P(d)
            L.fc1_w, L.fc1_b = P(cfg.encoder_ffn_dim, d), P(cfg.encoder_ffn_dim)
            L.fc2_w, L.fc2_b = P(d, cfg.encoder_ffn_dim), P(d)
            self.layers.append(L)
        self.ln_post_w, self.ln_post_b = P(d), P(d)
        self.proj1_w, self.proj1_b = P(d, d), P(d)
        self.proj2_w, self.proj2_b = P(cfg.output_dim, d), P(cfg.output_dim)
        self.register_buffer("pos", sinusoids(cfg.max_source_positions, d).to(device, dt), persistent=False)

    @torch.no_grad()
    def random_init_(self, seed: int = 0, std: float = 0.02):
        dev = self.conv1_w.device
        for idx, (n, p) in enumerate(self.named_parameters()):
            if n.endswith("_b"):
                p.zero_()
            elif "ln" in n:
                p.fill_(1.0)
            else:
                g = torch.Generator(device=dev).manual_seed(seed * 31337 + idx)
                p.normal_(0.0, std, generator=g)
        with torch.no_grad():
            self.conv1_w[:, 9:] = 0
        return self

    @torch.no_grad()
    def load_hf_state_dict(self, sd: dict[str, torch.Tensor]):
        """``thinker.audio_tower.*`` tensors with the prefix stripped."""
        cv = lambda w: w.permute(0, 2, 3, 1).reshape(w.shape[0], -1)  # noqa: E731  [O, C, kh, kw] -> [O, (kh, kw, c)]
        w1 = cv(sd["conv2d1.weight"])
        self.conv1_w.zero_()
        self.conv1_w[:, :w1.shape[1]] = w1
        self.conv1_b.copy_(sd["conv2d1.bias"])
        self.conv2_w.copy_(cv(sd["conv2d2.weight"]))
        self.conv2_b.copy_(sd["conv2d2.bias"])
        self.conv3_w.copy_(cv(sd["conv2d3.weight"]))
        self.conv3_b.copy_(sd["conv2d3.bias"])
        self.conv_out_w.copy_(sd["conv_out.weight"])
        for i, L in enumerate(self.layers):
            p = f"layers.{i}."
            L.ln1_w.copy_(sd[p + "self_attn_layer_norm.weight"])
            L.ln1_b.copy_(sd[p + "self_attn_layer_norm.bias"])
            L.qkv_w.copy_(torch.cat([sd[p + f"self_attn.{n}_proj.weight"] for n in "qkv"], 0))
            L.qkv_b.copy_(torch.cat([sd[p + f"self_attn.{n}_proj.bias"] for n in "qkv"], 0))
            L.o_w.copy_(sd[p + "self_attn.out_proj.weight"])
            L.o_b.copy_(sd[p + "self_attn.out_proj.bias"])
            L.ln2_w.copy_(sd[p + "final_layer_norm.weight"])
            L.ln2_b.copy_(sd[p + "final_layer_norm.bias"])
            L.fc1_w.copy_(sd[p + "fc1.weight"])
            L.fc1_b.copy_(sd[p + "fc1.bias"])
            L.fc2_w.copy_(sd[p + "fc2.weight"])
            L.fc2_b.copy_(sd[p + "fc2.bias"])
        self.ln_post_w.copy_(sd["ln_post.weight"])
        self.ln_post_b.copy_(sd["ln_post.bias"])
        self.proj1_w.copy_(sd["proj1.weight"])
        self.proj1_b.copy_(sd["proj1.bias"])
        self.proj2_w.copy_(sd["proj2.weight"])
        self.proj2_b.copy_(sd["proj2.bias"])

    def output_lengths(self, mel_lens: list[int]) -> list[int]:
        cs = 2 * self.cfg.n_window
        out = []
        for n in mel_lens:
            full, rem = divmod(n, cs)
            out.append(full * cnn_out_len(cs) + (cnn_out_len(rem) if rem else 0))
        return out

    @torch.no_grad()
    def forward(self, mels: list[torch.Tensor]) -> list[torch.Tensor]:
        """mels: list of [n_mel, T_i] -> list of [tokens_i, output_dim]."""
        cfg = self.cfg
        dev = self.conv1_w.device
        cs = 2 * cfg.n_window
        # every mel cut into chunks of cs frames (the last one zero padded): one pad + view per
        # request instead of one slice per chunk
        parts, valid = [], []
        for m in mels:
            T = m.shape[1]
            nc = (T + cs - 1) // cs
            mp = torch.nn.functional.pad(m, (0, nc * cs - T)) if nc * cs != T else m
            parts.append(mp.reshape(m.shape[0], nc, cs).permute(1, 0, 2))
            valid += [cnn_out_len(cs)] * (T // cs) + ([cnn_out_len(T % cs)] if T % cs else [])
        N = len(valid)
        x = torch.cat(parts, 0).to(dev, cfg.dtype).unsqueeze(-1).contiguous()  # [N, mel, cs, 1]
        if x.is_cuda:
            x = torch.nn.functional.pad(x, (0, 7))  # channel pad to 8 for 16-byte rows
            w1 = torch.nn.functional.pad(self.conv1_w.view(-1, 16)[:, :9].reshape(-1, 9, 1), (0, 7)).reshape(-1, 72)
            h = A.conv2d(x, w1, self.conv1_b, 3, 2, 1, act="gelu")
        else:
            h = A.conv2d(x, self.conv1_w[:, :9].contiguous(), self.conv1_b, 3, 2, 1, act="gelu")
        h = A.conv2d(h, self.conv2_w, self.conv2_b, 3, 2, 1, act="gelu")
        h = A.conv2d(h, self.conv3_w, self.conv3_b, 3, 2, 1, act="gelu")  # [N, F, t, C]
        Nn, F_, t, C = h.shape
        h = h.permute(0, 2, 3, 1).reshape(N * t, C * F_).contiguous()
        h = ops.linear(h, self.conv_out_w).view(N, t, -1)
        h = h + self.pos[:t].to(h.dtype)
        if all(v == t for v in valid):
            rows = h.reshape(N * t, -1)
        else:   # drop the padded tail tokens of partial chunks with one gather
            keep = np.concatenate([np.arange(v) + i * t for i, v in enumerate(valid)])
            rows = h.reshape(N * t, -1).index_select(0, torch.from_numpy(keep).to(dev))
        # attention windows: every request's tokens cut into windows of win tokens
        win = cnn_out_len(cs) * (cfg.n_window_infer // cs)
        per_req = self.output_lengths([m.shape[1] for m in mels])
        lens = []
        for n in per_req:
            lens += [win] * (n // win) + ([n % win] if n % win else [])
        cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=dev)
        d, nh = cfg.d_model, cfg.encoder_attention_heads
        hd = d // nh
        hs = rows
        for L in self.layers:
            n1 = ops.layer_norm(hs, L.ln1_w, L.ln1_b, 1e-5)
            qkv = ops.linear(n1, L.qkv_w, bias=L.qkv_b)
            if qkv.is_cuda:   # strided q / k / v views of the fused rows (the kernel takes row strides)
                q, k, v = qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:]
            else:
                q, k, v = qkv[:, :d].contiguous(), qkv[:, d:2 * d].contiguous(), qkv[:, 2 * d:].contiguous()
            a = ops.varlen_attention(q, k, v, cu, nh, nh, hd, q_lens=lens)
            hs = ops.linear(a, L.o_w, bias=L.o_b, residual=hs)
            n2 = ops.layer_norm(hs, L.ln2_w, L.ln2_b, 1e-5)
            f = ops.linear(n2, L.fc1_w, bias=L.fc1_b, act="gelu")
            hs = ops.linear(f, L.fc2_w, bias=L.fc2_b, residual=hs)
        hs = ops.layer_norm(hs, self.ln_post_w, self.ln_post_b, 1e-5)
        hs = ops.linear(hs, self.proj1_w, bias=self.proj1_b, act="gelu")
        hs = ops.linear(hs, self.proj2_w, bias=self.proj2_b)
        return list(torch.split(hs, per_req))
