"""S2-Pro codec (modded DAC, 44.1 kHz): code decoding on the sm_100a kernels and
reference-audio encoding.

Decoder path (``DACDecoder.decode``, channels-last, bf16):

  codes [B, 10, T] (semantic codebook 4096 + 9 residual codebooks of 1024)
  -> z = sum_c table_c[code_c]: each VQ's 1x1 ``out_proj`` is folded into its
     codebook at load time (table_c = codebook_c @ W_c^T + b_c), so RVQ decoding
     is one gather-sum kernel (``ops.vq_embed``) instead of 10 tiny GEMMs
  -> post_module: causal window-128 transformer, 8 layers x 1024 (16 x 64
     heads, SwiGLU 3072, pairwise RoPE, LayerScale folded into wo / w2)
  -> upsample x2 twice: ConvTranspose(k=2, s=2) as one GEMM + ConvNeXt block
  -> Decoder: causal conv k7 1024->1536, 4 blocks (Snake1d, causal
     ConvTranspose k=2s stride 8/8/4/2, residual units k7 dil 1/3/9 + k1),
     Snake1d, conv k7 96->1, tanh.   2048 samples per code frame.

Weight-normalised convolutions are resolved to plain weights at load time.
Reference: DAC / Decoder / DecoderBlock / ResidualUnit / WindowLimitedTransformer
(sglang_omni/models/fishaudio_s2_pro/fish_speech/models/dac/modded_dac.py:92-921)
and DownsampleResidualVectorQuantize.decode (.../dac/rvq.py:204-367), with the
configuration of .../fish_speech/configs/modded_dac_vq.yaml.

Encoder path (``DACEncoder``): audio -> codes for voice-cloning references.
The reference runs it on the CPU in preprocessing (pipeline/stages.py:193-215);
here it is plain PyTorch (fp32) on whichever device it is given.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from ... import ops
from ...ops import audio as A


@dataclass
class DACConfig:
    sample_rate: int = 44100
    latent_dim: int = 1024
    decoder_dim: int = 1536
    decoder_rates: tuple = (8, 8, 4, 2)
    encoder_dim: int = 64
    encoder_rates: tuple = (2, 4, 8, 8)
    encoder_transformer_layers: tuple = (0, 0, 0, 4)
    encoder_window: int = 512
    n_codebooks: int = 9
    codebook_size: int = 1024
    semantic_codebook_size: int = 4096
    codebook_dim: int = 8
    downsample_factor: tuple = (2, 2)
    tf_layers: int = 8
    tf_heads: int = 16
    tf_head_dim: int = 64
    tf_inter: int = 3072
    tf_window: int = 128
    rope_base: float = 10000.0
    norm_eps: float = 1e-5
    dtype: torch.dtype = torch.bfloat16

    @property
    def num_codebooks(self) -> int:
        return self.n_codebooks + 1

    @property
    def hop(self) -> int:
        return int(math.prod(self.decoder_rates) * math.prod(self.downsample_factor))

    @property
    def encoder_hop(self) -> int:
        return int(math.prod(self.encoder_rates))


# ----------------------------------------------------------------------------- checkpoint helpers
def wn_weight(sd: dict, prefix: str) -> torch.Tensor:
    """Effective weight of a (possibly weight-normalised) conv: g * v / ||v|| (norm over all dims but 0)."""
    if prefix + "weight" in sd:
        return sd[prefix + "weight"].float()
    if prefix + "parametrizations.weight.original0" in sd:
        g, v = sd[prefix + "parametrizations.weight.original0"], sd[prefix + "parametrizations.weight.original1"]
    else:
        g, v = sd[prefix + "weight_g"], sd[prefix + "weight_v"]
    v = v.float()
    n = v.flatten(1).norm(dim=1).view(-1, *([1] * (v.dim() - 1)))
    return g.float() * v / n


def _conv_rows(w: torch.Tensor) -> torch.Tensor:
    """Conv1d weight [O, I, K] -> GEMM rows [O, K*I] in (tap, channel) order."""
    return w.permute(0, 2, 1).reshape(w.shape[0], -1)


def _tconv_rows(w: torch.Tensor) -> torch.Tensor:
    """ConvTranspose1d weight [I, O, K] -> GEMM rows [K*O, I] in (tap, out channel) order."""
    return w.permute(2, 1, 0).reshape(-1, w.shape[0])


def _tf_keys(prefix: str, layers: int) -> list[str]:
    ks = [prefix + "norm.weight"]
    for i in range(layers):
        p = f"{prefix}layers.{i}."
        ks += [p + n for n in ("attention.wqkv.weight", "attention.wo.weight", "feed_forward.w1.weight",
                               "feed_forward.w3.weight", "feed_forward.w2.weight", "attention_norm.weight",
                               "ffn_norm.weight", "attention_layer_scale.gamma", "ffn_layer_scale.gamma")]
    return ks


def random_dac_state_dict(cfg: DACConfig = DACConfig(), seed: int = 0, std: float = 0.02,
                          encoder: bool = True) -> dict[str, torch.Tensor]:
    """A checkpoint-format state dict with random weights (weight norm as g / v pairs)."""
    g = torch.Generator().manual_seed(seed)
    sd: dict[str, torch.Tensor] = {}

    def rnd(*shape, s=std):
        return torch.randn(*shape, generator=g) * s

    def wn_conv(prefix, o, i, k, bias=True):
        v = rnd(o, i, k)
        sd[prefix + "parametrizations.weight.original1"] = v
        sd[prefix + "parametrizations.weight.original0"] = v.flatten(1).norm(dim=1).view(o, 1, 1) * (
            1.0 + 0.1 * torch.rand(o, 1, 1, generator=g))
        if bias:
            sd[prefix + "bias"] = rnd(o)

    def wn_tconv(prefix, i, o, k):
        v = rnd(i, o, k)
        sd[prefix + "parametrizations.weight.original1"] = v
        sd[prefix + "parametrizations.weight.original0"] = v.flatten(1).norm(dim=1).view(i, 1, 1)
        sd[prefix + "bias"] = rnd(o)

    def snake(prefix, c):
        sd[prefix + "alpha"] = 1.0 + 0.2 * torch.rand(1, c, 1, generator=g)

    def resunit(prefix, c, causal_k=7):
        snake(prefix + "block.0.", c)
        wn_conv(prefix + "block.1.conv.", c, c, causal_k)
        snake(prefix + "block.2.", c)
        wn_conv(prefix + "block.3.conv.", c, c, 1)

    def transformer(prefix, layers, dim, inter):
        sd[prefix + "norm.weight"] = 1.0 + 0.1 * rnd(dim, s=1.0)
        for i in range(layers):
            p = f"{prefix}layers.{i}."
            sd[p + "attention.wqkv.weight"] = rnd(3 * dim, dim)
            sd[p + "attention.wo.weight"] = rnd(dim, dim)
            sd[p + "feed_forward.w1.weight"] = rnd(inter, dim)
            sd[p + "feed_forward.w3.weight"] = rnd(inter, dim)
            sd[p + "feed_forward.w2.weight"] = rnd(dim, inter)
            sd[p + "attention_norm.weight"] = 1.0 + 0.1 * rnd(dim, s=1.0)
            sd[p + "ffn_norm.weight"] = 1.0 + 0.1 * rnd(dim, s=1.0)
            sd[p + "attention_layer_scale.gamma"] = torch.full((dim,), 0.5)
            sd[p + "ffn_layer_scale.gamma"] = torch.full((dim,), 0.5)

    def convnext(prefix, dim):
        sd[prefix + "dwconv.conv.weight"] = rnd(dim, 1, 7, s=0.2)
        sd[prefix + "dwconv.conv.bias"] = rnd(dim)
        sd[prefix + "norm.weight"] = 1.0 + 0.1 * rnd(dim, s=1.0)
        sd[prefix + "norm.bias"] = rnd(dim)
        sd[prefix + "pwconv1.weight"] = rnd(4 * dim, dim)
        sd[prefix + "pwconv1.bias"] = rnd(4 * dim)
        sd[prefix + "pwconv2.weight"] = rnd(dim, 4 * dim)
        sd[prefix + "pwconv2.bias"] = rnd(dim)
        sd[prefix + "gamma"] = torch.full((dim,), 0.5)

    D = cfg.latent_dim
    q = "quantizer."
    for name, n, size in (("semantic_quantizer.", 1, cfg.semantic_codebook_size),
                          ("quantizer.", cfg.n_codebooks, cfg.codebook_size)):
        for i in range(n):
            p = f"{q}{name}quantizers.{i}."
            sd[p + "codebook.weight"] = rnd(size, cfg.codebook_dim, s=1.0)
            wn_conv(p + "in_proj.", cfg.codebook_dim, D, 1)
            wn_conv(p + "out_proj.", D, cfg.codebook_dim, 1)
    transformer(q + "post_module.", cfg.tf_layers, D, cfg.tf_inter)
    transformer(q + "pre_module.", cfg.tf_layers, D, cfg.tf_inter)
    for j, f in enumerate(cfg.downsample_factor):
        sd[f"{q}downsample.{j}.0.conv.weight"] = rnd(D, D, f)
        sd[f"{q}downsample.{j}.0.conv.bias"] = rnd(D)
        convnext(f"{q}downsample.{j}.1.", D)
        sd[f"{q}upsample.{j}.0.conv.weight"] = rnd(D, D, f)
        sd[f"{q}upsample.{j}.0.conv.bias"] = rnd(D)
        convnext(f"{q}upsample.{j}.1.", D)
    # decoder
    ch = cfg.decoder_dim
    wn_conv("decoder.model.0.conv.", ch, D, 7)
    for i, s in enumerate(cfg.decoder_rates):
        cin, cout = ch // 2 ** i, ch // 2 ** (i + 1)
        p = f"decoder.model.{i + 1}.block."
        snake(p + "0.", cin)
        wn_tconv(p + "1.conv.", cin, cout, 2 * s)
        for r in range(3):
            resunit(f"{p}{r + 2}.", cout)
    n = len(cfg.decoder_rates) + 1
    snake(f"decoder.model.{n}.", ch // 2 ** len(cfg.decoder_rates))
    wn_conv(f"decoder.model.{n + 1}.conv.", 1, ch // 2 ** len(cfg.decoder_rates), 7)
    if encoder:
        d = cfg.encoder_dim
        wn_conv("encoder.block.0.conv.", d, 1, 7)
        for i, (s, nt) in enumerate(zip(cfg.encoder_rates, cfg.encoder_transformer_layers)):
            d *= 2
            p = f"encoder.block.{i + 1}.block."
            for r in range(3):
                resunit(f"{p}{r}.", d // 2)
            snake(p + "3.", d // 2)
            wn_conv(p + "4.conv.", d, d // 2, 2 * s)
            if nt:
                transformer(p + "5.", nt, d, 3 * d)
        n = len(cfg.encoder_rates) + 1
        snake(f"encoder.block.{n}.", d)
        wn_conv(f"encoder.block.{n + 1}.conv.", D, d, 3)
    return sd


# ----------------------------------------------------------------------------- decoder (GPU path)
class DACDecoder(nn.Module):
    def __init__(self, cfg: DACConfig = DACConfig(), device="cpu"):
        super().__init__()
        self.cfg = cfg
        dt = cfg.dtype
        D = cfg.latent_dim
        P = lambda *s, dtype=dt: nn.Parameter(torch.zeros(*s, dtype=dtype, device=device),  # noqa: E731
                                              requires_grad=False)
        nq = cfg.num_codebooks
        self.cb_rows = max(cfg.semantic_codebook_size, cfg.codebook_size)
        self.rvq_table = P(nq * self.cb_rows, D)
        self.zero_row = P(1, D)
        self.tf = nn.ModuleList()
        for _ in range(cfg.tf_layers):
            L = nn.Module()
            L.ln1, L.ln2 = P(D), P(D)
            L.qkv = P(3 * D, D)
            L.o = P(D, D)
            L.w13 = P(2 * cfg.tf_inter, D)
            L.w2 = P(D, cfg.tf_inter)
            self.tf.append(L)
        self.tf_norm = P(D)
        self.up = nn.ModuleList()
        for f in reversed(cfg.downsample_factor):
            U = nn.Module()
            U.f = f
            U.tconv_w, U.tconv_b = P(f * D, D), P(D)
            U.dw_w, U.dw_b = P(D, 7, dtype=torch.float32), P(D, dtype=torch.float32)
            U.ln_w, U.ln_b = P(D), P(D)
            U.pw1_w, U.pw1_b = P(4 * D, D), P(4 * D)
            U.pw2_w, U.pw2_b = P(D, 4 * D), P(D)
            self.up.append(U)
        ch = cfg.decoder_dim
        self.conv_in_w, self.conv_in_b = P(ch, 7 * D), P(ch)
        self.blocks = nn.ModuleList()
        for i, s in enumerate(cfg.decoder_rates):
            cin, cout = ch // 2 ** i, ch // 2 ** (i + 1)
            Bk = nn.Module()
            Bk.stride = s
            Bk.alpha = P(cin, dtype=torch.float32)
            Bk.tconv_w, Bk.tconv_b = P(2 * s * cout, cin), P(cout)
            Bk.units = nn.ModuleList()
            for dil in (1, 3, 9):
                Un = nn.Module()
                Un.dil = dil
                Un.a1, Un.a2 = P(cout, dtype=torch.float32), P(cout, dtype=torch.float32)
                Un.c1_w, Un.c1_b = P(cout, 7 * cout), P(cout)
                Un.c2_w, Un.c2_b = P(cout, cout), P(cout)
                Bk.units.append(Un)
            self.blocks.append(Bk)
        cl = ch // 2 ** len(cfg.decoder_rates)
        self.out_alpha = P(cl, dtype=torch.float32)
        self.conv_out_w, self.conv_out_b = P(1, 7 * cl), P(1)
        cos, sin = ops.rope_tables(cfg.tf_head_dim, cfg.rope_base, 1 << 15, device, round_bf16=True)
        self.register_buffer("cos_tab", cos, persistent=False)
        self.register_buffer("sin_tab", sin, persistent=False)

    @torch.no_grad()
    def load_state_dict_dac(self, sd: dict[str, torch.Tensor]):
        cfg = self.cfg
        cp = lambda dst, src: dst.copy_(src.to(dst.dtype).reshape(dst.shape))  # noqa: E731
        q = "quantizer."
        self.rvq_table.zero_()
        tabs = []
        for name, n in (("semantic_quantizer.", 1), ("quantizer.", cfg.n_codebooks)):
            for i in range(n):
                p = f"{q}{name}quantizers.{i}."
                w = wn_weight(sd, p + "out_proj.")[:, :, 0]                  # [D, cb_dim]
                tabs.append(sd[p + "codebook.weight"].float() @ w.t() + sd[p + "out_proj.bias"].float())
        for c, t in enumerate(tabs):
            self.rvq_table[c * self.cb_rows: c * self.cb_rows + t.shape[0]].copy_(t.to(self.rvq_table.dtype))
        pm = q + "post_module."
        for i, L in enumerate(self.tf):
            p = f"{pm}layers.{i}."
            ga = sd[p + "attention_layer_scale.gamma"].float()
            gf = sd[p + "ffn_layer_scale.gamma"].float()
            cp(L.ln1, sd[p + "attention_norm.weight"])
            cp(L.ln2, sd[p + "ffn_norm.weight"])
            cp(L.qkv, sd[p + "attention.wqkv.weight"])
            cp(L.o, sd[p + "attention.wo.weight"].float() * ga[:, None])
            cp(L.w13, torch.cat([sd[p + "feed_forward.w1.weight"], sd[p + "feed_forward.w3.weight"]], 0))
            cp(L.w2, sd[p + "feed_forward.w2.weight"].float() * gf[:, None])
        cp(self.tf_norm, sd[pm + "norm.weight"])
        nd = len(cfg.downsample_factor)
        for k, U in enumerate(self.up):
            j = nd - 1 - k                      # upsample modules run in reverse index order
            p = f"{q}upsample.{j}."
            cp(U.tconv_w, _tconv_rows(sd[p + "0.conv.weight"].float()))
            cp(U.tconv_b, sd[p + "0.conv.bias"])
            cp(U.dw_w, sd[p + "1.dwconv.conv.weight"].float()[:, 0])
            cp(U.dw_b, sd[p + "1.dwconv.conv.bias"])
            cp(U.ln_w, sd[p + "1.norm.weight"])
            cp(U.ln_b, sd[p + "1.norm.bias"])
            cp(U.pw1_w, sd[p + "1.pwconv1.weight"])
            cp(U.pw1_b, sd[p + "1.pwconv1.bias"])
            gm = sd[p + "1.gamma"].float()
            cp(U.pw2_w, sd[p + "1.pwconv2.weight"].float() * gm[:, None])
            cp(U.pw2_b, sd[p + "1.pwconv2.bias"].float() * gm)
        cp(self.conv_in_w, _conv_rows(wn_weight(sd, "decoder.model.0.conv.")))
        cp(self.conv_in_b, sd["decoder.model.0.conv.bias"])
        for i, Bk in enumerate(self.blocks):
            p = f"decoder.model.{i + 1}.block."
            cp(Bk.alpha, sd[p + "0.alpha"])
            cp(Bk.tconv_w, _tconv_rows(wn_weight(sd, p + "1.conv.")))
            cp(Bk.tconv_b, sd[p + "1.conv.bias"])
            for r, Un in enumerate(Bk.units):
                u = f"{p}{r + 2}.block."
                cp(Un.a1, sd[u + "0.alpha"])
                cp(Un.c1_w, _conv_rows(wn_weight(sd, u + "1.conv.")))
                cp(Un.c1_b, sd[u + "1.conv.bias"])
                cp(Un.a2, sd[u + "2.alpha"])
                cp(Un.c2_w, _conv_rows(wn_weight(sd, u + "3.conv.")))
                cp(Un.c2_b, sd[u + "3.conv.bias"])
        n = len(cfg.decoder_rates) + 1
        cp(self.out_alpha, sd[f"decoder.model.{n}.alpha"])
        cp(self.conv_out_w, _conv_rows(wn_weight(sd, f"decoder.model.{n + 1}.conv.")))
        cp(self.conv_out_b, sd[f"decoder.model.{n + 1}.conv.bias"])
        return self

    # ------------------------------------------------------------------ forward pieces
    def _rvq(self, codes: torch.Tensor) -> torch.Tensor:
        """codes [B, 10, T] -> z rows [B*T, D] (sum of the folded codebook tables)."""
        cfg = self.cfg
        B, Q, T = codes.shape
        c = codes.to(torch.int32).clone()
        c[:, 0].clamp_(0, cfg.semantic_codebook_size - 1)
        c[:, 1:].clamp_(0, cfg.codebook_size - 1)
        rows = c.permute(0, 2, 1).reshape(B * T, Q).contiguous()
        n = B * T
        dev = codes.device
        return ops.vq_embed(self.zero_row, self.rvq_table, rows, self.cb_rows, 1.0, 0, -1,
                            ids=torch.zeros(n, dtype=torch.int32, device=dev),
                            code_row=torch.arange(n, dtype=torch.int32, device=dev))

    def _transformer(self, h: torch.Tensor, B: int, T: int) -> torch.Tensor:
        cfg = self.cfg
        nh, hd = cfg.tf_heads, cfg.tf_head_dim
        D = nh * hd
        pos = torch.arange(T, dtype=torch.int32, device=h.device).repeat(B)
        cu = torch.arange(0, (B + 1) * T, T, dtype=torch.int32, device=h.device)
        for L in self.tf:
            n1 = ops.rms_norm(h, L.ln1, cfg.norm_eps)
            qkv = ops.linear(n1, L.qkv)
            ops.qkv_rope_store(qkv, nh, nh, hd, pos, self.cos_tab, self.sin_tab, hd, None, None, cfg.norm_eps,
                               False)
            q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
            if qkv.is_cuda:
                a = ops.varlen_attention(q, k, v, cu, nh, nh, hd, causal=True, window=cfg.tf_window, q_lens=[T] * B)
            else:
                a = ops.varlen_attention(q.contiguous(), k.contiguous(), v.contiguous(), cu, nh, nh, hd, causal=True,
                                         window=cfg.tf_window)
            h = ops.linear(a, L.o, residual=h)
            n2 = ops.rms_norm(h, L.ln2, cfg.norm_eps)
            h = ops.linear(ops.linear(n2, L.w13, gated=True), L.w2, residual=h)
        return ops.rms_norm(h, self.tf_norm, cfg.norm_eps)

    @torch.no_grad()
    def decode(self, codes: torch.Tensor) -> torch.Tensor:
        """codes [B, 10, T] int -> waveform [B, T * hop] float32 in [-1, 1]."""
        cfg = self.cfg
        B, _, T = codes.shape
        D = cfg.latent_dim
        x = self._transformer(self._rvq(codes), B, T).view(B, T, D)
        for U in self.up:
            Tc = x.shape[1]
            y = ops.linear(x.reshape(B * Tc, D), U.tconv_w, out_dtype=torch.float32)  # [B*T, f*D]
            x = (y.view(B, Tc, U.f, D) + U.tconv_b.float()).reshape(B, Tc * U.f, D).to(cfg.dtype)
            inp = x
            h = A.dwconv1d_causal(x, U.dw_w, U.dw_b)
            h = ops.layer_norm(h, U.ln_w, U.ln_b, 1e-6)
            h = ops.linear(h, U.pw1_w, bias=U.pw1_b, act="gelu")
            x = ops.linear(h, U.pw2_w, bias=U.pw2_b, residual=inp)
        x = A.causal_conv1d(x, self.conv_in_w, self.conv_in_b, 7)
        for Bk in self.blocks:
            x = A.snake(x, Bk.alpha, None, log_scale=False)
            Tn = x.shape[1]
            x = A.conv_transpose1d(x, Bk.tconv_w, Bk.tconv_b, Bk.stride, trim_left=0, t_out=Tn * Bk.stride)
            for Un in Bk.units:
                h = A.snake(x, Un.a1, None, log_scale=False)
                h = A.causal_conv1d(h, Un.c1_w, Un.c1_b, 7, dilation=Un.dil)
                h = A.snake(h, Un.a2, None, log_scale=False)
                x = A.causal_conv1d(h, Un.c2_w, Un.c2_b, 1, residual=x)
        x = A.snake(x, self.out_alpha, None, log_scale=False)
        wav = A.causal_conv1d(x, self.conv_out_w, self.conv_out_b, 7)
        return torch.tanh(wav.float().reshape(B, -1))


# ----------------------------------------------------------------------------- encoder (reference audio)
def _rms(x, w, eps):
    return (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)) * w


def _rope_pairs(x: torch.Tensor, base: float) -> torch.Tensor:
    """Pairwise RoPE over [B, T, H, D] with positions 0..T-1 (bf16-rounded tables)."""
    B, T, H, D = x.shape
    inv = 1.0 / (base ** (torch.arange(0, D, 2, device=x.device)[: D // 2].float() / D))
    ang = torch.arange(T, device=x.device).float()[:, None] * inv[None]
    c, s = ang.cos().bfloat16().float(), ang.sin().bfloat16().float()
    xr = x.float().view(B, T, H, D // 2, 2)
    c, s = c[None, :, None], s[None, :, None]
    out = torch.stack([xr[..., 0] * c - xr[..., 1] * s, xr[..., 1] * c + xr[..., 0] * s], -1)
    return out.flatten(3)


def window_transformer_ref(x: torch.Tensor, sd: dict, prefix: str, layers: int, heads: int, window: int,
                           base: float = 10000.0, eps: float = 1e-5) -> torch.Tensor:
    """fp32 WindowLimitedTransformer (causal, channels-first [B, C, T] in and out)."""
    h = x.transpose(1, 2).float()
    B, T, D = h.shape
    hd = D // heads
    i = torch.arange(T, device=x.device)
    mask = (i[None, :] <= i[:, None]) & (i[None, :] > i[:, None] - window)
    for li in range(layers):
        p = f"{prefix}layers.{li}."
        n1 = _rms(h, sd[p + "attention_norm.weight"].float(), eps)
        q, k, v = (n1 @ sd[p + "attention.wqkv.weight"].float().t()).split(D, -1)
        q = _rope_pairs(q.view(B, T, heads, hd), base).transpose(1, 2)
        k = _rope_pairs(k.view(B, T, heads, hd), base).transpose(1, 2)
        v = v.view(B, T, heads, hd).transpose(1, 2)
        a = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        a = a.transpose(1, 2).reshape(B, T, D) @ sd[p + "attention.wo.weight"].float().t()
        h = h + a * sd[p + "attention_layer_scale.gamma"].float()
        n2 = _rms(h, sd[p + "ffn_norm.weight"].float(), eps)
        f = F.silu(n2 @ sd[p + "feed_forward.w1.weight"].float().t()) * (n2 @ sd[p + "feed_forward.w3.weight"].float().t())
        h = h + (f @ sd[p + "feed_forward.w2.weight"].float().t()) * sd[p + "ffn_layer_scale.gamma"].float()
    h = _rms(h, sd[prefix + "norm.weight"].float(), eps)
    return h.transpose(1, 2)


def snake_ref(x, alpha):
    a = alpha.float().view(1, -1, 1)
    return x + (a + 1e-9).reciprocal() * torch.sin(a * x).pow(2)


def causal_conv_ref(x, w, b, stride=1, dilation=1):
    """CausalConvNet: left pad (k_eff - stride), right pad so the last partial frame is produced."""
    k_eff = (w.shape[-1] - 1) * dilation + 1
    pad = k_eff - stride
    n_frames = (x.shape[-1] - k_eff + pad) / stride + 1
    ideal = (math.ceil(n_frames) - 1) * stride + (k_eff - pad)
    extra = ideal - x.shape[-1]
    x = F.pad(x, (pad, extra))
    return F.conv1d(x, w, b, stride=stride, dilation=dilation)


def convnext_ref(x, sd, p):
    C = x.shape[1]
    w = sd[p + "dwconv.conv.weight"].float()                                    # [C, 1, 7], depthwise
    h = F.conv1d(F.pad(x, (w.shape[-1] - 1, 0)), w, sd[p + "dwconv.conv.bias"].float(), groups=C)
    h = h.transpose(1, 2)
    h = F.layer_norm(h, (C,), sd[p + "norm.weight"].float(), sd[p + "norm.bias"].float(), 1e-6)
    h = F.gelu(h @ sd[p + "pwconv1.weight"].float().t() + sd[p + "pwconv1.bias"].float())
    h = (h @ sd[p + "pwconv2.weight"].float().t() + sd[p + "pwconv2.bias"].float()) * sd[p + "gamma"].float()
    return x + h.transpose(1, 2)


def resunit_ref(x, sd, p, dil):
    y = snake_ref(x, sd[p + "block.0.alpha"])
    y = causal_conv_ref(y, wn_weight(sd, p + "block.1.conv."), sd[p + "block.1.conv.bias"].float(), dilation=dil)
    y = snake_ref(y, sd[p + "block.2.alpha"])
    y = F.conv1d(y, wn_weight(sd, p + "block.3.conv."), sd[p + "block.3.conv.bias"].float())
    return x[..., : y.shape[-1]] + y


class DACEncoder:
    """Audio [B, N] at 44.1 kHz -> codes [B, 10, ceil(N / 2048)] (fp32 PyTorch)."""

    def __init__(self, sd: dict[str, torch.Tensor], cfg: DACConfig = DACConfig(), device="cpu"):
        self.cfg = cfg
        self.sd = {k: v.to(device, torch.float32) for k, v in sd.items()
                   if k.startswith(("encoder.", "quantizer."))}
        self.device = torch.device(device)

    def _conv(self, x, prefix, stride=1, dilation=1):
        return causal_conv_ref(x, wn_weight(self.sd, prefix), self.sd[prefix + "bias"], stride, dilation)

    @torch.no_grad()
    def encode(self, audio: torch.Tensor) -> torch.Tensor:
        cfg, sd = self.cfg, self.sd
        x = audio.to(self.device, torch.float32)
        if x.dim() == 1:
            x = x[None]
        frame = cfg.encoder_hop * 4
        n = x.shape[-1]
        x = F.pad(x, (0, math.ceil(n / frame) * frame - n))[:, None]
        x = self._conv(x, "encoder.block.0.conv.")
        d = cfg.encoder_dim
        for i, (s, nt) in enumerate(zip(cfg.encoder_rates, cfg.encoder_transformer_layers)):
            d *= 2
            p = f"encoder.block.{i + 1}.block."
            for r, dil in enumerate((1, 3, 9)):
                x = resunit_ref(x, sd, f"{p}{r}.", dil)
            x = snake_ref(x, sd[p + "3.alpha"])
            x = self._conv(x, p + "4.conv.", stride=s)
            if nt:
                x = window_transformer_ref(x, sd, p + "5.", nt, d // 64, cfg.encoder_window, cfg.rope_base,
                                           cfg.norm_eps)
        n = len(cfg.encoder_rates) + 1
        x = snake_ref(x, sd[f"encoder.block.{n}.alpha"])
        z = self._conv(x, f"encoder.block.{n + 1}.conv.")
        q = "quantizer."
        for j, f in enumerate(cfg.downsample_factor):
            z = causal_conv_ref(z, sd[f"{q}downsample.{j}.0.conv.weight"], sd[f"{q}downsample.{j}.0.conv.bias"], f)
            z = convnext_ref(z, sd, f"{q}downsample.{j}.1.")
        z = window_transformer_ref(z, sd, q + "pre_module.", cfg.tf_layers, cfg.tf_heads, cfg.tf_window,
                                   cfg.rope_base, cfg.norm_eps)
        codes = []
        res = z
        for name, n in (("semantic_quantizer.", 1), ("quantizer.", cfg.n_codebooks)):
            if name == "quantizer.":
                res = z - zq_sem
            for i in range(n):
                p = f"{q}{name}quantizers.{i}."
                ze = F.conv1d(res, wn_weight(sd, p + "in_proj."), sd[p + "in_proj.bias"])     # [B, 8, T]
                e = F.normalize(ze.transpose(1, 2), dim=-1)                                    # [B, T, 8]
                cb = F.normalize(sd[p + "codebook.weight"], dim=-1)                            # [K, 8]
                idx = (e @ cb.t()).argmax(-1)                                                  # nearest on the sphere
                zq = F.conv1d(sd[p + "codebook.weight"][idx].transpose(1, 2), wn_weight(sd, p + "out_proj."),
                              sd[p + "out_proj.bias"])
                codes.append(idx)
                if name == "semantic_quantizer.":
                    zq_sem = zq
                else:
                    res = res - zq
        return torch.stack(codes, 1)


def dac_decode_reference(sd: dict[str, torch.Tensor], codes: torch.Tensor, cfg: DACConfig = DACConfig()) -> torch.Tensor:
    """fp32 PyTorch decode straight from a checkpoint-format state dict (the oracle of DACDecoder)."""
    sd = {k: v.float() for k, v in sd.items() if k.startswith(("decoder.", "quantizer."))}
    codes = codes.long().clone()
    codes[:, 0].clamp_(max=cfg.semantic_codebook_size - 1)
    codes[:, 1:].clamp_(max=cfg.codebook_size - 1)
    q = "quantizer."
    z = 0
    for c, (name, i) in enumerate([("semantic_quantizer.", 0)] + [("quantizer.", i) for i in range(cfg.n_codebooks)]):
        p = f"{q}{name}quantizers.{i}."
        zp = sd[p + "codebook.weight"][codes[:, c]].transpose(1, 2)              # [B, 8, T]
        z = z + F.conv1d(zp, wn_weight(sd, p + "out_proj."), sd[p + "out_proj.bias"])
    z = window_transformer_ref(z, sd, q + "post_module.", cfg.tf_layers, cfg.tf_heads, cfg.tf_window, cfg.rope_base,
                               cfg.norm_eps)
    for j in reversed(range(len(cfg.downsample_factor))):
        p = f"{q}upsample.{j}."
        z = F.conv_transpose1d(z, sd[p + "0.conv.weight"], sd[p + "0.conv.bias"], stride=cfg.downsample_factor[j])
        z = convnext_ref(z, sd, p + "1.")
    x = causal_conv_ref(z, wn_weight(sd, "decoder.model.0.conv."), sd["decoder.model.0.conv.bias"])
    for i, s in enumerate(cfg.decoder_rates):
        p = f"decoder.model.{i + 1}.block."
        x = snake_ref(x, sd[p + "0.alpha"])
        y = F.conv_transpose1d(x, wn_weight(sd, p + "1.conv."), sd[p + "1.conv.bias"], stride=s)
        x = y[..., : y.shape[-1] - s]
        for r, dil in enumerate((1, 3, 9)):
            x = resunit_ref(x, sd, f"{p}{r + 2}.", dil)
    n = len(cfg.decoder_rates) + 1
    x = snake_ref(x, sd[f"decoder.model.{n}.alpha"])
    x = causal_conv_ref(x, wn_weight(sd, f"decoder.model.{n + 1}.conv."), sd[f"decoder.model.{n + 1}.conv.bias"])
    return torch.tanh(x)[:, 0]
