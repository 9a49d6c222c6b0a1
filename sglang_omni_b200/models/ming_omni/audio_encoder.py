"""Ming-Omni audio tower on the sm_100a kernels: Whisper encoder + projection.

  mel [128, T] -> conv k3 p1 (128 -> 1280) + GELU -> conv k3 s2 p1 + GELU
  -> + sinusoidal positions -> 32 x [LN, MHA (20 x 64, full attention over the
  segment), LN, GELU MLP 4x] -> LN
  -> projection: conv k3 s2 p1 (1280 -> 4096), then (mlp_depth - 1) x [GELU, Linear]
  -> L2-normalised rows (``norm_query_embeds``).

Convolutions run as im2col + tcgen05 GEMMs (bias + GELU in the epilogue), the
segments of a batch go through one varlen attention launch per layer.
Reference: MingAudioEncoder (sglang_omni/models/ming_omni/components/audio_encoder.py:35-200),
which runs openai-whisper's AudioEncoder; checkpoint keys ``audio.*`` and
``linear_proj_audio.*``.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from ... import ops
from ...ops import audio as A
from .hf_config import WhisperConfig


def sinusoids(length: int, channels: int, max_timescale: float = 10000.0) -> torch.Tensor:
    """[length, channels]: sin of position * geometric frequencies, then cos (Transformer positional code)."""
    half = channels // 2
    inc = math.log(max_timescale) / (half - 1)
    inv = torch.exp(-inc * torch.arange(half, dtype=torch.float32))
    t = torch.arange(length, dtype=torch.float32)[:, None] * inv[None, :]
    return torch.cat([t.sin(), t.cos()], 1)


class MingAudioEncoder(nn.Module):
    def __init__(self, cfg: WhisperConfig = WhisperConfig(), device="cpu", dtype=torch.bfloat16):
        super().__init__()
        self.cfg = cfg
        D, M = cfg.n_state, cfg.n_mels
        P = lambda *s: nn.Parameter(torch.empty(*s, dtype=dtype, device=device), requires_grad=False)  # noqa: E731
        self.dtype = dtype
        self.conv1_w, self.conv1_b = P(D, 3 * M), P(D)           # GEMM rows [O, (tap, channel)]
        self.conv2_w, self.conv2_b = P(D, 3 * D), P(D)
        self.register_buffer("pos", sinusoids(cfg.n_ctx, D).to(device, dtype), persistent=False)
        self.blocks = nn.ModuleList()
        for _ in range(cfg.n_layer):
            B = nn.Module()
            B.ln1_w, B.ln1_b = P(D), P(D)
            B.qkv_w, B.qkv_b = P(3 * D, D), P(3 * D)                 # key has no bias: zeros
            B.o_w, B.o_b = P(D, D), P(D)
            B.ln2_w, B.ln2_b = P(D), P(D)
            B.fc1_w, B.fc1_b = P(4 * D, D), P(4 * D)
            B.fc2_w, B.fc2_b = P(D, 4 * D), P(D)
            self.blocks.append(B)
        self.ln_post_w, self.ln_post_b = P(D), P(D)
        O = cfg.out_dim
        self.proj_w, self.proj_b = P(O, cfg.ds_kernel_size * D), P(O)
        self.mlp = nn.ModuleList()
        for _ in range(1, cfg.mlp_depth):
            L = nn.Module()
            L.w, L.b = P(O, O), P(O)
            self.mlp.append(L)

    @torch.no_grad()
    def random_init_(self, seed: int = 0, std: float = 0.02):
        g = torch.Generator(device=self.conv1_w.device).manual_seed(seed)
        for name, p in self.named_parameters():
            if "ln" in name and name.endswith("_w"):
                p.fill_(1.0)
            elif name.endswith(("_b", ".b")):
                p.zero_()
            else:
                p.normal_(0.0, std, generator=g)
        return self

    @torch.no_grad()
    def load_hf_state_dict(self, sd: dict[str, torch.Tensor]):
        """Keys relative to the checkpoint root (``audio.*``, ``linear_proj_audio.*``)."""
        c = lambda dst, src: dst.copy_(src.to(dst.dtype).reshape(dst.shape))  # noqa: E731
        rows = lambda w: w.permute(0, 2, 1).reshape(w.shape[0], -1)  # noqa: E731  [O, I, K] -> [O, (K, I)]
        c(self.conv1_w, rows(sd["audio.conv1.weight"]))
        c(self.conv1_b, sd["audio.conv1.bias"])
        c(self.conv2_w, rows(sd["audio.conv2.weight"]))
        c(self.conv2_b, sd["audio.conv2.bias"])
        if "audio.positional_embedding" in sd:
            n = min(self.pos.shape[0], sd["audio.positional_embedding"].shape[0])
            self.pos[:n].copy_(sd["audio.positional_embedding"][:n].to(self.pos.dtype))
        D = self.cfg.n_state
        for i, B in enumerate(self.blocks):
            p = f"audio.blocks.{i}."
            c(B.ln1_w, sd[p + "attn_ln.weight"])
            c(B.ln1_b, sd[p + "attn_ln.bias"])
            c(B.qkv_w, torch.cat([sd[p + "attn.query.weight"], sd[p + "attn.key.weight"],
                                  sd[p + "attn.value.weight"]], 0))
            c(B.qkv_b, torch.cat([sd[p + "attn.query.bias"], torch.zeros(D, dtype=sd[p + "attn.query.bias"].dtype),
                                  sd[p + "attn.value.bias"]], 0))
            c(B.o_w, sd[p + "attn.out.weight"])
            c(B.o_b, sd[p + "attn.out.bias"])
            c(B.ln2_w, sd[p + "mlp_ln.weight"])
            c(B.ln2_b, sd[p + "mlp_ln.bias"])
            c(B.fc1_w, sd[p + "mlp.0.weight"])
            c(B.fc1_b, sd[p + "mlp.0.bias"])
            c(B.fc2_w, sd[p + "mlp.2.weight"])
            c(B.fc2_b, sd[p + "mlp.2.bias"])
        c(self.ln_post_w, sd["audio.ln_post.weight"])
        c(self.ln_post_b, sd["audio.ln_post.bias"])
        c(self.proj_w, rows(sd["linear_proj_audio.0.weight"]))
        c(self.proj_b, sd["linear_proj_audio.0.bias"])
        for j, L in enumerate(self.mlp):
            k = f"linear_proj_audio.{3 * j + 3}."       # Sequential: conv, transpose, [GELU, Linear]...
            c(L.w, sd[k + "weight"])
            c(L.b, sd[k + "bias"])
        return self

    def output_length(self, mel_frames: int) -> int:
        n = (mel_frames - 1) // 2 + 1
        k, s = self.cfg.ds_kernel_size, self.cfg.ds_stride
        return (n - k + 2 * (k // 2)) // s + 1

    @torch.no_grad()
    def forward(self, mels: list[torch.Tensor]) -> list[torch.Tensor]:
        """mels: list of [n_mels, T_i] -> list of [tokens_i, out_dim]."""
        cfg = self.cfg
        D, nh = cfg.n_state, cfg.n_head
        hd = D // nh
        outs1 = []
        for m in mels:   # per segment: the convolutions are length-dependent
            x = m.t().to(self.conv1_w.device, self.dtype).contiguous()[None]           # [1, T, n_mels]
            T = x.shape[1]
            h = A.causal_conv1d(x, self.conv1_w, self.conv1_b, 3, pad_left=1, t_out=T, act="gelu")
            T2 = (T - 1) // 2 + 1
            h = A.causal_conv1d(h, self.conv2_w, self.conv2_b, 3, stride=2, pad_left=1, t_out=T2, act="gelu")[0]
            outs1.append(h + self.pos[:T2])
        lens = [o.shape[0] for o in outs1]
        hs = torch.cat(outs1, 0)
        dev = hs.device
        cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device=dev)
        for B in self.blocks:
            n1 = ops.layer_norm(hs, B.ln1_w, B.ln1_b, 1e-5)
            qkv = ops.linear(n1, B.qkv_w, bias=B.qkv_b)
            q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
            if qkv.is_cuda:
                a = ops.varlen_attention(q, k, v, cu, nh, nh, hd, q_lens=lens)
            else:
                a = ops.varlen_attention(q.contiguous(), k.contiguous(), v.contiguous(), cu, nh, nh, hd)
            hs = ops.linear(a, B.o_w, bias=B.o_b, residual=hs)
            n2 = ops.layer_norm(hs, B.ln2_w, B.ln2_b, 1e-5)
            hs = ops.linear(ops.linear(n2, B.fc1_w, bias=B.fc1_b, act="gelu"), B.fc2_w, bias=B.fc2_b, residual=hs)
        hs = ops.layer_norm(hs, self.ln_post_w, self.ln_post_b, 1e-5)
        res = []
        o = 0
        k, s = cfg.ds_kernel_size, cfg.ds_stride
        for n in lens:
            seg = hs[o:o + n][None]
            o += n
            t_out = (n - k + 2 * (k // 2)) // s + 1
            y = A.causal_conv1d(seg.contiguous(), self.proj_w, self.proj_b, k, stride=s, pad_left=k // 2,
                                t_out=t_out)[0]
            for L in self.mlp:
                y = ops.linear(_gelu(y), L.w, bias=L.b)    # GELU of the conv output, then Linear
            if cfg.norm_query_embeds:
                y = F.normalize(y.float(), dim=-1).to(y.dtype)
            res.append(y)
        return res


def _gelu(x: torch.Tensor) -> torch.Tensor:
    return F.gelu(x.float()).to(x.dtype)
