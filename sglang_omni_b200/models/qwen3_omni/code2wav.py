"""Qwen3-Omni Code2Wav: 16-codebook codes (12.5 Hz) -> 24 kHz waveform.

codes [B, 16, T] -> mean of the 16 code embeddings -> 8-layer causal
sliding-window (72) transformer with LayerScale -> 2 x (kernel=stride=2
transposed conv + ConvNeXt) -> causal conv 1024->1536 k7 -> 4 decoder blocks
(SnakeBeta, transposed conv kernel 2r stride r, 3 residual units with dilated
k7 causal convs) -> SnakeBeta -> conv ->1 k7 -> clamp(-1, 1).  1920 samples
per frame.

Everything is channels-last; convolutions are tcgen05 GEMMs over im2col rows,
SnakeBeta / depthwise conv / overlap-add are the kernels in csrc/audio_ops.cu,
the transformer uses the varlen sliding-window attention kernel.  ConvNeXt's
``gamma`` is folded into pwconv2 at load.

Streaming (``StreamingCode2Wav``): every ``chunk`` new frames the model runs on
``left_context + chunk`` frames of each stream, batched across streams, and
emits the samples after the context, like the reference executor
(sglang_omni/models/qwen3_omni/components/code2wav_executor.py:54-265, chunk
10, context 25).  Architecture: transformers Qwen3OmniMoeCode2Wav.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
from torch import nn

from ... import ops
from ...ops import audio as A


@dataclass
class Code2WavConfig:
    codebook_size: int = 2048
    hidden_size: int = 1024
    num_heads: int = 16
    num_kv_heads: int = 16
    sliding_window: int = 72
    intermediate_size: int = 3072
    layer_scale_initial_scale: float = 0.01
    rms_norm_eps: float = 1e-5
    num_layers: int = 8
    num_quantizers: int = 16
    upsample_rates: tuple = (8, 5, 4, 3)
    upsampling_ratios: tuple = (2, 2)
    decoder_dim: int = 1536
    rope_theta: float = 10000.0
    max_position: int = 8000
    dtype: torch.dtype = torch.bfloat16

    @property
    def head_dim(self):
        return self.hidden_size // self.num_heads

    @property
    def total_upsample(self):
        return int(math.prod(self.upsample_rates) * math.prod(self.upsampling_ratios))


class Code2Wav(nn.Module):
    def __init__(self, cfg: Code2WavConfig, device="cpu"):
        super().__init__()
        self.cfg = cfg
        H, dt = cfg.hidden_size, cfg.dtype
        P = lambda *s, d=dt: nn.Parameter(torch.empty(*s, dtype=d, device=device), requires_grad=False)  # noqa
        F32 = torch.float32
        self.code_embedding = P(cfg.codebook_size * cfg.num_quantizers, H)
        self.layers = nn.ModuleList()
        for _ in range(cfg.num_layers):
            L = nn.Module()
            L.ln1, L.ln2 = P(H), P(H)
            L.qkv = P(3 * H if cfg.num_kv_heads == cfg.num_heads else H + 2 * cfg.num_kv_heads * cfg.head_dim, H)
            L.o = P(H, H)
            L.mlp13 = P(2 * cfg.intermediate_size, H)
            L.mlp2 = P(H, cfg.intermediate_size)
            L.attn_scale, L.mlp_scale = P(H), P(H)
            self.layers.append(L)
        self.final_norm = P(H)
        self.up = nn.ModuleList()
        for f in cfg.upsampling_ratios:
            U = nn.Module()
            U.tconv_w = P(f * H, H)        # kernel == stride: [(j, o), c]
            U.tconv_b = P(H)
            U.dw_w = P(H, 7, d=F32)
            U.dw_b = P(H, d=F32)
            U.ln_w, U.ln_b = P(H), P(H)
            U.pw1_w, U.pw1_b = P(4 * H, H), P(4 * H)
            U.pw2_w, U.pw2_b = P(H, 4 * H), P(H)  # gamma folded in
            self.up.append(U)
        D = cfg.decoder_dim
        self.conv_in_w, self.conv_in_b = P(D, 7 * H), P(D)
        self.blocks = nn.ModuleList()
        for i, r in enumerate(cfg.upsample_rates):
            cin, cout = D // 2 ** i, D // 2 ** (i + 1)
            Bk = nn.Module()
            Bk.snake_a, Bk.snake_b = P(cin, d=F32), P(cin, d=F32)
            Bk.tconv_w, Bk.tconv_b = P(2 * r * cout, cin), P(cout)
            Bk.units = nn.ModuleList()
            for dil in (1, 3, 9):
                Un = nn.Module()
                Un.dil = dil
                Un.a1, Un.b1 = P(cout, d=F32), P(cout, d=F32)
                Un.c1_w, Un.c1_b = P(cout, 7 * cout), P(cout)
                Un.a2, Un.b2 = P(cout, d=F32), P(cout, d=F32)
                Un.c2_w, Un.c2_b = P(cout, cout), P(cout)
                Bk.units.append(Un)
            self.blocks.append(Bk)
        cl = D // 2 ** len(cfg.upsample_rates)
        self.out_snake_a, self.out_snake_b = P(cl, d=F32), P(cl, d=F32)
        self.conv_out_w, self.conv_out_b = P(1, 7 * cl), P(1)
        cos, sin = ops.rope_tables(cfg.head_dim, cfg.rope_theta, cfg.max_position, device,
                                   round_bf16=cfg.dtype == torch.bfloat16)
        self.register_buffer("cos_tab", cos, persistent=False)
        self.register_buffer("sin_tab", sin, persistent=False)
        self.register_buffer("code_offset", torch.arange(cfg.num_quantizers, device=device) * cfg.codebook_size,
                             persistent=False)

    @torch.no_grad()
    def random_init_(self, seed: int = 0, std: float = 0.02):
        dev = self.code_embedding.device
        for idx, (name, p) in enumerate(self.named_parameters()):
            leaf = name.rsplit(".", 1)[-1]
            if leaf in ("ln1", "ln2", "final_norm", "ln_w"):
                p.fill_(1.0)
            elif leaf in ("attn_scale", "mlp_scale"):
                p.fill_(self.cfg.layer_scale_initial_scale)
            elif leaf.startswith(("snake", "a", "b")) and p.dtype == torch.float32 and p.dim() == 1:
                p.zero_()
            elif leaf.endswith("_b") or leaf == "ln_b":
                p.zero_()
            else:
                g = torch.Generator(device=dev).manual_seed(seed * 7919 + idx)
                p.normal_(0.0, std, generator=g)
        return self

    # ------------------------------------------------------------------ load from HF names
    @torch.no_grad()
    def load_hf_state_dict(self, sd: dict[str, torch.Tensor]):
        """Loads ``code2wav.*`` checkpoint tensors (prefix already stripped)."""
        cfg = self.cfg
        g = lambda k: sd[k]  # noqa: E731
        self.code_embedding.copy_(g("code_embedding.weight"))
        for i, L in enumerate(self.layers):
            p = f"pre_transformer.layers.{i}."
            L.ln1.copy_(g(p + "input_layernorm.weight"))
            L.ln2.copy_(g(p + "post_attention_layernorm.weight"))
            L.qkv.copy_(torch.cat([g(p + f"self_attn.{n}_proj.weight") for n in "qkv"], 0))
            L.o.copy_(g(p + "self_attn.o_proj.weight"))
            L.mlp13.copy_(torch.cat([g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")], 0))
            L.mlp2.copy_(g(p + "mlp.down_proj.weight"))
            L.attn_scale.copy_(g(p + "self_attn_layer_scale.scale"))
            L.mlp_scale.copy_(g(p + "mlp_layer_scale.scale"))
        self.final_norm.copy_(g("pre_transformer.norm.weight"))
        for i, U in enumerate(self.up):
            p = f"upsample.{i}."
            w = g(p + "0.conv.weight")  # [Cin, Cout, K]
            U.tconv_w.copy_(w.permute(2, 1, 0).reshape(-1, w.shape[0]))
            U.tconv_b.copy_(g(p + "0.conv.bias"))
            U.dw_w.copy_(g(p + "1.dwconv.conv.weight").squeeze(1))
            U.dw_b.copy_(g(p + "1.dwconv.conv.bias"))
            U.ln_w.copy_(g(p + "1.norm.weight"))
            U.ln_b.copy_(g(p + "1.norm.bias"))
            U.pw1_w.copy_(g(p + "1.pwconv1.weight"))
            U.pw1_b.copy_(g(p + "1.pwconv1.bias"))
            gamma = g(p + "1.gamma").float()
            U.pw2_w.copy_((g(p + "1.pwconv2.weight").float() * gamma[:, None]))
            U.pw2_b.copy_((g(p + "1.pwconv2.bias").float() * gamma))
        conv2d = lambda w: w.permute(0, 2, 1).reshape(w.shape[0], -1)  # noqa: E731  [O, I, K] -> [O, (K, I)]
        self.conv_in_w.copy_(conv2d(g("decoder.0.conv.weight")))
        self.conv_in_b.copy_(g("decoder.0.conv.bias"))
        for i, Bk in enumerate(self.blocks):
            p = f"decoder.{i + 1}.block."
            Bk.snake_a.copy_(g(p + "0.alpha"))
            Bk.snake_b.copy_(g(p + "0.beta"))
            w = g(p + "1.conv.weight")
            Bk.tconv_w.copy_(w.permute(2, 1, 0).reshape(-1, w.shape[0]))
            Bk.tconv_b.copy_(g(p + "1.conv.bias"))
            for j, Un in enumerate(Bk.units):
                q = p + f"{j + 2}."
                Un.a1.copy_(g(q + "act1.alpha"))
                Un.b1.copy_(g(q + "act1.beta"))
                Un.c1_w.copy_(conv2d(g(q + "conv1.conv.weight")))
                Un.c1_b.copy_(g(q + "conv1.conv.bias"))
                Un.a2.copy_(g(q + "act2.alpha"))
                Un.b2.copy_(g(q + "act2.beta"))
                Un.c2_w.copy_(conv2d(g(q + "conv2.conv.weight")))
                Un.c2_b.copy_(g(q + "conv2.conv.bias"))
        n = len(cfg.upsample_rates) + 1
        self.out_snake_a.copy_(g(f"decoder.{n}.alpha"))
        self.out_snake_b.copy_(g(f"decoder.{n}.beta"))
        self.conv_out_w.copy_(conv2d(g(f"decoder.{n + 1}.conv.weight")))
        self.conv_out_b.copy_(g(f"decoder.{n + 1}.conv.bias"))

    # ------------------------------------------------------------------ forward
    def make_aux(self, B: int, T: int, device) -> dict:
        """Device-side index tensors of a [B, T] window batch (positions, sequence offsets,
        attention tiles), built once per shape so a captured forward does no host copies."""
        from ...ops.attention import prefill_tiles

        cfg = self.cfg
        req, tok0 = prefill_tiles([T] * B, cfg.num_heads // cfg.num_kv_heads)
        return {"pos": torch.arange(T, dtype=torch.int32, device=device).repeat(B),
                "cu": torch.arange(0, (B + 1) * T, T, dtype=torch.int32, device=device),
                "tiles": (torch.tensor(req, dtype=torch.int32, device=device),
                          torch.tensor(tok0, dtype=torch.int32, device=device))}

    def _transformer(self, x: torch.Tensor, B: int, T: int, aux: dict | None = None) -> torch.Tensor:
        cfg = self.cfg
        H, nh, nkv, hd = cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        if aux is not None:
            pos, cu, tiles = aux["pos"], aux["cu"], aux["tiles"]
        else:
            pos = torch.arange(T, dtype=torch.int32, device=x.device).repeat(B)
            cu = torch.arange(0, (B + 1) * T, T, dtype=torch.int32, device=x.device)
            tiles = None
        h = x
        for L in self.layers:
            n1 = ops.rms_norm(h, L.ln1, cfg.rms_norm_eps)
            qkv = ops.linear(n1, L.qkv)
            ops.qkv_rope_store(qkv, nh, nkv, hd, pos, self.cos_tab, self.sin_tab, hd, None, None,
                               cfg.rms_norm_eps, True, None, True, None, None, None)
            q = qkv[:, : nh * hd]
            k = qkv[:, nh * hd:(nh + nkv) * hd]
            v = qkv[:, (nh + nkv) * hd:]
            if qkv.is_cuda:
                attn = ops.varlen_attention(q, k, v, cu, nh, nkv, hd, causal=True, window=cfg.sliding_window,
                                            q_lens=[T] * B, tiles=tiles)
            else:
                attn = ops.varlen_attention(q.contiguous(), k.contiguous(), v.contiguous(), cu, nh, nkv, hd,
                                            causal=True, window=cfg.sliding_window)
            a = ops.linear(attn, L.o)
            h = h + (a.float() * L.attn_scale.float()).to(h.dtype)
            n2 = ops.rms_norm(h, L.ln2, cfg.rms_norm_eps)
            m = ops.linear(ops.linear(n2, L.mlp13, gated=True), L.mlp2)
            h = h + (m.float() * L.mlp_scale.float()).to(h.dtype)
        return ops.rms_norm(h, self.final_norm, cfg.rms_norm_eps)

    def forward(self, codes: torch.Tensor, aux: dict | None = None) -> torch.Tensor:
        """codes [B, Q, T] int -> waveform [B, T * total_upsample] float32 (``aux``: ``make_aux``)."""
        cfg = self.cfg
        B, Q, T = codes.shape
        idx = (codes.long() + self.code_offset.view(1, -1, 1)).permute(0, 2, 1)  # [B, T, Q]
        x = self.code_embedding[idx].float().mean(2).to(cfg.dtype).reshape(B * T, cfg.hidden_size)
        x = self._transformer(x, B, T, aux).view(B, T, cfg.hidden_size)
        for f, U in zip(cfg.upsampling_ratios, self.up):
            Tc = x.shape[1]
            y = ops.linear(x.contiguous(), U.tconv_w)  # [B, T, f*C]
            x = (y.view(B, Tc, f, -1) + U.tconv_b).reshape(B, Tc * f, -1).to(cfg.dtype)
            inp = x
            h = A.dwconv1d_causal(x, U.dw_w, U.dw_b)
            h = ops.layer_norm(h, U.ln_w, U.ln_b, 1e-6)
            h = ops.linear(h, U.pw1_w, bias=U.pw1_b, act="gelu")
            x = ops.linear(h, U.pw2_w, bias=U.pw2_b, residual=inp)
        x = A.causal_conv1d(x, self.conv_in_w, self.conv_in_b, 7)
        for r, Bk in zip(cfg.upsample_rates, self.blocks):
            x = A.snake(x, Bk.snake_a, Bk.snake_b)
            x = A.conv_transpose1d(x, Bk.tconv_w, Bk.tconv_b, r)
            for Un in Bk.units:
                res = x
                h = A.snake(x, Un.a1, Un.b1)
                h = A.causal_conv1d(h, Un.c1_w, Un.c1_b, 7, dilation=Un.dil)
                h = A.snake(h, Un.a2, Un.b2)
                x = A.causal_conv1d(h, Un.c2_w, Un.c2_b, 1, residual=res)
        x = A.snake(x, self.out_snake_a, self.out_snake_b)
        wav = A.causal_conv1d(x, self.conv_out_w, self.conv_out_b, 7)
        return wav.float().reshape(B, -1).clamp(-1.0, 1.0)


class Code2WavGraphs:
    """CUDA graphs of the vocoder forward, one per (batch bucket, window length).

    A streaming chunk runs ~150 kernels; launched from Python in a process whose
    thinker and talker threads hold the interpreter between their own launches,
    that costs far more than the GPU time.  A replay is one launch.  Batches are
    padded to the next bucket (padding rows decode code 0 and are dropped);
    windows that were not captured (final flushes of odd length) run eagerly.
    The returned rows view the graph's output buffer: read them before the same
    (bucket, window) graph replays again."""

    BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128)

    def __init__(self, model: "Code2Wav", max_batch: int = 32):
        self.model = model
        self.max_batch = max_batch
        self.graphs: dict[tuple[int, int], tuple] = {}
        self._pool = None

    @torch.no_grad()
    def capture(self, B: int, W: int) -> None:
        """Captured in the thread-local mode on a private stream (other stages' threads keep
        running their GPU work meanwhile)."""
        from ...utils.cuda_graph import capture_graph

        m = self.model
        dev = m.code_embedding.device
        codes = torch.zeros(B, m.cfg.num_quantizers, W, dtype=torch.long, device=dev)
        aux = m.make_aux(B, W, dev)
        with torch.cuda.device(dev):
            g, out = capture_graph(lambda: m(codes, aux), warmup=1, pool=self._pool)
        self._pool = g.pool()
        self.graphs[(B, W)] = (g, codes, aux, out)

    def capture_windows(self, windows, max_batch: int | None = None) -> None:
        top = max_batch or self.max_batch
        for W in sorted(set(windows)):
            for B in self.BUCKETS:
                if B > top:
                    break
                if (B, W) not in self.graphs:
                    self.capture(B, W)

    @torch.no_grad()
    def __call__(self, codes: torch.Tensor) -> torch.Tensor:
        B, _, W = codes.shape
        Bb = next((b for b in self.BUCKETS if b >= B), None)
        hit = self.graphs.get((Bb, W)) if Bb is not None else None
        if hit is None:
            return self.model(codes)
        g, buf, _, out = hit
        buf[:B].copy_(codes, non_blocking=True)
        if B < Bb:
            buf[B:].zero_()
        g.replay()
        return out[:B]


def chunk_windows(chunk: int, left_context: int, first_chunk: int) -> list[int]:
    """Window lengths (context + new frames) of a stream's successive full chunks."""
    out, emitted = [], 0
    while True:
        new = first_chunk if emitted == 0 else chunk
        w = min(left_context, emitted) + new
        if w in out:
            return out
        out.append(w)
        emitted += new


@dataclass
class _StreamState:
    codes: list = field(default_factory=list)   # list of [Q] code columns
    emitted_frames: int = 0


class StreamingCode2Wav:
    """Incremental decoding of many streams: every ``chunk`` new frames (or at
    the end) each ready stream decodes ``context + new`` frames; ready streams
    with equal window length are batched into one forward."""

    def __init__(self, model: Code2Wav, chunk: int = 10, left_context: int = 25, first_chunk: int | None = None,
                 graphs: Code2WavGraphs | None = None):
        self.model = model
        self.chunk = chunk
        self.left_context = left_context
        self.first_chunk = first_chunk or chunk
        self.streams: dict[str, _StreamState] = {}
        self.graphs = graphs
        self._pinned: torch.Tensor | None = None

    def windows(self) -> list[int]:
        return chunk_windows(self.chunk, self.left_context, self.first_chunk)

    def capture_graphs(self) -> None:
        if self.graphs is not None:
            self.graphs.capture_windows(self.windows())

    def add_codes(self, rid: str, codes: torch.Tensor) -> None:
        """codes: [Q] or [T, Q] frames for stream rid."""
        st = self.streams.setdefault(rid, _StreamState())
        if codes.dim() == 1:
            codes = codes.unsqueeze(0)
        st.codes.extend(list(codes))

    def ready(self, rid: str, final: bool = False) -> bool:
        st = self.streams.get(rid)
        if st is None:
            return False
        pending = len(st.codes) - st.emitted_frames
        need = self.first_chunk if st.emitted_frames == 0 else self.chunk
        return pending >= need or (final and pending > 0)

    @torch.no_grad()
    def decode_ready(self, rids: list[str], final: bool = False, finals=None,
                     to_host: bool = False) -> dict[str, torch.Tensor]:
        """Returns {rid: float32 waveform of the new frames} for every ready stream.

        ``final`` (all streams) or ``finals`` (a set of stream ids) flush the streams
        whose last frame has arrived.  ``to_host``: numpy arrays, copied with one
        device-to-host transfer per window group on the current stream."""
        up = self.model.cfg.total_upsample
        groups: dict[tuple[int, int], list[tuple[str, torch.Tensor]]] = {}
        for rid in rids:
            fin = final or (finals is not None and rid in finals)
            if not self.ready(rid, fin):
                continue
            st = self.streams[rid]
            pending = len(st.codes) - st.emitted_frames
            if fin:
                end = len(st.codes)
            elif st.emitted_frames == 0:
                end = self.first_chunk + (pending - self.first_chunk) // self.chunk * self.chunk
            else:
                end = st.emitted_frames + pending // self.chunk * self.chunk
            ctx = min(self.left_context, st.emitted_frames)
            window = torch.stack(st.codes[st.emitted_frames - ctx:end], 1)  # [Q, W]
            groups.setdefault((window.shape[1], ctx), []).append((rid, window))
            st.emitted_frames = end
        out = {}
        dev = self.model.code_embedding.device
        run = self.graphs if self.graphs is not None and dev.type == "cuda" else self.model
        for (W, ctx), items in groups.items():
            codes = torch.stack([w for _, w in items], 0).to(dev, non_blocking=True)
            wav = run(codes)
            if to_host and wav.is_cuda:
                n = wav[:, ctx * up:]
                if self._pinned is None or self._pinned.numel() < n.numel():
                    self._pinned = torch.empty(max(n.numel(), 1 << 20), dtype=torch.float32, pin_memory=True)
                host = self._pinned[:n.numel()].view(n.shape)
                host.copy_(n, non_blocking=True)
                torch.cuda.current_stream(dev).synchronize()
                for (rid, _), wv in zip(items, host):
                    out[rid] = wv.numpy().copy()
            elif to_host:
                for (rid, _), wv in zip(items, wav):
                    out[rid] = wv[ctx * up:].float().numpy().copy()
            else:
                for (rid, _), wv in zip(items, wav):
                    out[rid] = wv[ctx * up:]
        return out

    def close(self, rid: str) -> None:
        self.streams.pop(rid, None)
