"""Stateful streaming Code2Wav: every chunk runs only its new frames.

The windowed decoder (``code2wav.StreamingCode2Wav``; the reference executor,
sglang_omni/models/qwen3_omni/components/code2wav_executor.py:211-232, works
the same way) re-runs ``left_context`` (25) frames in front of every 10-frame
chunk and keeps the samples after them.  This decoder instead keeps, per
stream, what the next chunk needs from the past:

* the sliding-window transformer's keys and values (after RoPE) in a ring of
  KV pages per stream and layer, read by the paged prefill attention kernel
  with the window limit; positions are the stream's absolute frame indices;
* for every causal convolution, its last (K - 1) * dilation input samples;
* for every decoder-block transposed convolution (kernel 2r, stride r, trimmed
  by r on both sides, so output block j needs input samples j and j + 1), its
  last input sample.

The concatenated chunks of a stream equal the full-sequence forward of all of
its frames (``Code2Wav.forward``).  The windowed decoder only approximates that
(its context is cut at 25 frames) and loses the trimmed tail samples of every
chunk.  The first chunk of a stream yields W * 1920 - d samples, where d is the
one-input look-ahead of the transposed convs carried through the upsampling
(555 samples at 24 kHz for the released sizes); every later chunk of W frames
yields exactly W * 1920 samples, the held-back ones coming out with it.

A steady chunk costs ``chunk`` frames of transformer and decoder work instead
of ``left_context + chunk``.  Shapes of a step depend only on (batch, frames,
first chunk or not): the per-stream state is selected on the device by slot
ids, so a step replays as one CUDA graph per (batch bucket, frames, first).
"""
from __future__ import annotations

import math

import torch

from ... import ops
from ...ops import audio as A
from ...ops.attention import prefill_attention
from ..common.stream_state import ConvHistory, KVRing, SlotStreams, StepGraphs, step_aux
from .code2wav import Code2Wav


def conv_history(model: Code2Wav) -> list[tuple[int, int]]:
    """(input samples kept, channels) of every stateful convolution, in forward order."""
    H = model.cfg.hidden_size
    out = [(U.dw_w.shape[1] - 1, H) for U in model.up]
    out.append((6, H))                                   # conv_in, kernel 7
    for Bk in model.blocks:
        out.append((1, Bk.snake_a.shape[0]))             # transposed conv: one input sample
        for Un in Bk.units:
            out.append((6 * Un.dil, Bk.tconv_b.shape[0]))  # kernel 7, dilation dil
    out.append((6, model.out_snake_a.shape[0]))          # conv_out, kernel 7
    return out


def first_chunk_samples(model: Code2Wav, frames: int) -> int:
    """Samples of a stream's first chunk of ``frames`` frames (the full-sequence length)."""
    n = frames * int(math.prod(model.cfg.upsampling_ratios))
    for r in model.cfg.upsample_rates:
        n = (n - 1) * r
    return max(n, 0)


class Code2WavStreamState:
    """Per-slot streaming state of one Code2Wav model and the chunk step over it.

    Slots 0 .. max_streams - 1 hold streams; slot ``max_streams`` is the sink of padding
    rows.  ``max_frames``: longest stream (RoPE table rows and block-table width).
    ``max_step``: most frames one step may carry (sets the KV ring depth)."""

    def __init__(self, model: Code2Wav, max_streams: int, max_frames: int = 16384, max_step: int = 64):
        cfg = model.cfg
        self.model = model
        self.device = model.code_embedding.device
        self.sink = max_streams
        self.max_frames = max_frames
        self.max_step = max_step
        S = max_streams + 1
        self.kv = KVRing(len(model.layers), cfg.num_kv_heads, cfg.head_dim, cfg.sliding_window, max_step, S,
                         max_frames, cfg.rope_theta, cfg.dtype, self.device,
                         round_bf16=cfg.dtype == torch.bfloat16)
        self.pos = torch.zeros(S, dtype=torch.int32, device=self.device)
        self.hist = ConvHistory(conv_history(model), S, cfg.dtype, self.device)

    def state_bytes(self) -> int:
        t = self.kv.tensors() + self.hist.t + [self.pos]
        return sum(x.numel() * x.element_size() for x in t)

    def make_aux(self, B: int, W: int) -> dict:
        cfg = self.model.cfg
        return step_aux(B, W, cfg.num_heads // cfg.num_kv_heads, self.device)

    def _transformer(self, x: torch.Tensor, slots: torch.Tensor, p0: torch.Tensor, aux: dict) -> torch.Tensor:
        m, cfg = self.model, self.model.cfg
        nh, nkv, hd = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        positions, slot_map, kv_lens, bt = self.kv.plan(slots, p0, aux["offs"])
        h = x
        for li, L in enumerate(m.layers):
            n1 = ops.rms_norm(h, L.ln1, cfg.rms_norm_eps)
            qkv = ops.linear(n1, L.qkv)
            ops.qkv_rope_store(qkv, nh, nkv, hd, positions, self.kv.cos, self.kv.sin, hd, None, None,
                               cfg.rms_norm_eps, True, None, True, slot_map, self.kv.k[li], self.kv.v[li])
            attn = prefill_attention(qkv[:, : nh * hd], self.kv.k[li], self.kv.v[li], bt, aux["cu"], kv_lens,
                                     aux["tiles"][0], aux["tiles"][1], nh, nkv, hd, causal=True,
                                     window=cfg.sliding_window)
            a = ops.linear(attn, L.o)
            h = h + (a.float() * L.attn_scale.float()).to(h.dtype)
            n2 = ops.rms_norm(h, L.ln2, cfg.rms_norm_eps)
            mm = ops.linear(ops.linear(n2, L.mlp13, gated=True), L.mlp2)
            h = h + (mm.float() * L.mlp_scale.float()).to(h.dtype)
        return ops.rms_norm(h, m.final_norm, cfg.rms_norm_eps)

    @torch.no_grad()
    def step(self, codes: torch.Tensor, slots: torch.Tensor, fresh: bool, aux: dict | None = None) -> torch.Tensor:
        """codes [B, Q, W] and slots [B] (int64) on the model's device -> float32 waveform rows
        [B, samples]: W * upsample samples per row, ``first_chunk_samples`` when ``fresh`` (every
        row is the first chunk of a new stream in its slot).  Advances every slot's state."""
        m, cfg = self.model, self.model.cfg
        B, _, W = codes.shape
        if W > self.max_step:
            raise ValueError(f"code2wav step of {W} frames > max_step {self.max_step}")
        aux = aux if aux is not None else self.make_aux(B, W)
        H = cfg.hidden_size
        hist = self.hist
        idx = (codes.long() + m.code_offset.view(1, -1, 1)).permute(0, 2, 1)
        x = m.code_embedding[idx].float().mean(2).to(cfg.dtype).reshape(B * W, H)
        p0 = torch.zeros(B, dtype=torch.int32, device=x.device) if fresh else self.pos.index_select(0, slots)
        x = self._transformer(x, slots, p0, aux).view(B, W, H)
        # the sink slot stays at frame 0, however many padding rows pass through it
        self.pos.index_copy_(0, slots, torch.where(slots == self.sink, 0, p0 + W).to(torch.int32))
        ci = 0
        for f, U in zip(cfg.upsampling_ratios, m.up):
            Tc = x.shape[1]
            y = ops.linear(x.contiguous(), U.tconv_w)
            x = (y.view(B, Tc, f, -1) + U.tconv_b).reshape(B, Tc * f, -1).to(cfg.dtype)
            inp = x
            xf = hist.extend(ci, x, slots, fresh)
            ci += 1
            h = A.dwconv1d_causal(xf, U.dw_w, U.dw_b)[:, xf.shape[1] - x.shape[1]:].contiguous()
            h = ops.layer_norm(h, U.ln_w, U.ln_b, 1e-6)
            h = ops.linear(h, U.pw1_w, bias=U.pw1_b, act="gelu")
            x = ops.linear(h, U.pw2_w, bias=U.pw2_b, residual=inp)
        xf = hist.extend(ci, x, slots, fresh)
        ci += 1
        x = A.causal_conv1d(xf, m.conv_in_w, m.conv_in_b, 7, pad_left=0, t_out=x.shape[1])
        for r, Bk in zip(cfg.upsample_rates, m.blocks):
            s = A.snake(x, Bk.snake_a, Bk.snake_b)
            if fresh:     # no earlier input: the trimmed output starts at block 0
                hist.keep_last(ci, s, slots)
                x = A.conv_transpose1d(s, Bk.tconv_w, Bk.tconv_b, r)
            else:         # the kept sample completes the block the previous chunk held back
                x = A.conv_transpose1d(hist.extend(ci, s, slots, False), Bk.tconv_w, Bk.tconv_b, r)
            ci += 1
            for Un in Bk.units:
                res = x
                h = A.snake(x, Un.a1, Un.b1)
                hf = hist.extend(ci, h, slots, fresh)
                ci += 1
                h = A.causal_conv1d(hf, Un.c1_w, Un.c1_b, 7, dilation=Un.dil, pad_left=0, t_out=h.shape[1])
                h = A.snake(h, Un.a2, Un.b2)
                x = A.causal_conv1d(h, Un.c2_w, Un.c2_b, 1, residual=res)
        s = A.snake(x, m.out_snake_a, m.out_snake_b)
        sf = hist.extend(ci, s, slots, fresh)
        wav = A.causal_conv1d(sf, m.conv_out_w, m.conv_out_b, 7, pad_left=0, t_out=s.shape[1])
        return wav.float().reshape(B, -1).clamp(-1.0, 1.0)


def StatefulGraphs(state: Code2WavStreamState, max_batch: int = 32) -> StepGraphs:
    """CUDA graphs of ``Code2WavStreamState.step`` per (batch bucket, frames, first chunk)."""
    return StepGraphs(state, state.model.cfg.num_quantizers, max_batch)


class StatefulStreamingCode2Wav(SlotStreams):
    """Incremental decoding of many Code2Wav streams with kept state (same interface as
    ``code2wav.StreamingCode2Wav``): every ``chunk`` new frames (or at the end) each ready
    stream decodes only its new frames.  ``max_streams`` open streams, ``max_frames`` frames
    per stream."""

    def __init__(self, model: Code2Wav, chunk: int = 10, first_chunk: int | None = None, max_streams: int = 32,
                 max_frames: int = 16384, use_graphs: bool = True):
        # a step carries one chunk, or what is left of a stream (less than a chunk) at its end
        state = Code2WavStreamState(model, max_streams, max_frames, max(chunk, first_chunk or chunk))
        graphs = StatefulGraphs(state, max_streams) if use_graphs and state.device.type == "cuda" else None
        super().__init__(state, chunk, first_chunk, graphs)
        self.model = model
