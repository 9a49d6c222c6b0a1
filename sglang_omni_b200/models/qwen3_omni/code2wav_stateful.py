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
from dataclasses import dataclass, field

import numpy as np
import torch

from ... import ops
from ...ops import audio as A
from ...ops.attention import PAGE, prefill_attention, prefill_tiles
from .code2wav import Code2Wav


def conv_history(model: Code2Wav) -> list[tuple[int, int]]:
    """(input samples kept, channels) of every stateful convolution, in forward order."""
    cfg = model.cfg
    H = cfg.hidden_size
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

    Slots 0 .. max_streams - 1 hold streams; slot ``max_streams`` is a sink that
    the padding rows of a graph bucket use (its contents are never read back).
    ``max_frames``: longest stream (RoPE table rows and block-table width).
    ``max_step``: most frames one step may carry (sets the KV ring depth)."""

    def __init__(self, model: Code2Wav, max_streams: int, max_frames: int = 16384, max_step: int = 64):
        cfg = model.cfg
        dev = model.code_embedding.device
        self.model = model
        self.S = max_streams + 1
        self.sink = max_streams
        self.max_frames = max_frames
        self.max_step = max_step
        # keys a step can need: window - 1 before its first frame, plus its own frames
        self.ring = -(-(cfg.sliding_window - 1 + max_step) // PAGE) + 1
        kv = (self.S * self.ring, cfg.num_kv_heads, PAGE, cfg.head_dim)
        self.k_cache = [torch.zeros(kv, dtype=cfg.dtype, device=dev) for _ in model.layers]
        self.v_cache = [torch.zeros(kv, dtype=cfg.dtype, device=dev) for _ in model.layers]
        nbt = -(-max_frames // PAGE)
        s = torch.arange(self.S, device=dev)[:, None]
        self.block_table = (s * self.ring + torch.arange(nbt, device=dev)[None] % self.ring).to(torch.int32)
        self.pos = torch.zeros(self.S, dtype=torch.int32, device=dev)
        self.cos, self.sin = ops.rope_tables(cfg.head_dim, cfg.rope_theta, max_frames, dev,
                                             round_bf16=cfg.dtype == torch.bfloat16)
        self.conv = [torch.zeros(self.S, n, c, dtype=cfg.dtype, device=dev) for n, c in conv_history(model)]

    def state_bytes(self) -> int:
        t = self.k_cache + self.v_cache + self.conv + [self.block_table, self.pos, self.cos, self.sin]
        return sum(x.numel() * x.element_size() for x in t)

    def make_aux(self, B: int, W: int) -> dict:
        """Device tensors of a [B, W] step that depend only on its shape (built once per shape)."""
        cfg = self.model.cfg
        dev = self.pos.device
        req, tok0 = prefill_tiles([W] * B, cfg.num_heads // cfg.num_kv_heads, 64)
        return {"offs": torch.arange(W, dtype=torch.int32, device=dev),
                "cu": torch.arange(0, (B + 1) * W, W, dtype=torch.int32, device=dev),
                "tiles": (torch.tensor(req, dtype=torch.int32, device=dev),
                          torch.tensor(tok0, dtype=torch.int32, device=dev))}

    def _history(self, i: int, x: torch.Tensor, slots: torch.Tensor, fresh: bool) -> torch.Tensor:
        """[kept input samples of conv i; x] per stream, and the new kept samples stored.  A
        stream's first chunk starts from zeros (the convolution's causal padding)."""
        st = self.conv[i]
        n = st.shape[1]
        B = x.shape[0]
        prev = x.new_zeros(B, n, x.shape[2]) if fresh else st.index_select(0, slots)
        xf = torch.cat([prev, x], 1)
        st.index_copy_(0, slots, xf[:, xf.shape[1] - n:])
        return xf

    def _keep_last(self, i: int, x: torch.Tensor, slots: torch.Tensor) -> None:
        st = self.conv[i]
        st.index_copy_(0, slots, x[:, x.shape[1] - st.shape[1]:])

    def _transformer(self, x: torch.Tensor, slots: torch.Tensor, p0: torch.Tensor, B: int, W: int,
                     aux: dict) -> torch.Tensor:
        m, cfg = self.model, self.model.cfg
        nh, nkv, hd = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        pos2 = p0.view(B, 1) + aux["offs"].view(1, W)                       # absolute frame index
        positions = pos2.reshape(-1)
        page = slots.view(B, 1) * self.ring + torch.div(pos2, PAGE, rounding_mode="floor") % self.ring
        slot_map = (page * PAGE + pos2 % PAGE).reshape(-1).to(torch.int32)
        kv_lens = (p0 + W).to(torch.int32)
        bt = self.block_table.index_select(0, slots)
        h = x
        for li, L in enumerate(m.layers):
            n1 = ops.rms_norm(h, L.ln1, cfg.rms_norm_eps)
            qkv = ops.linear(n1, L.qkv)
            ops.qkv_rope_store(qkv, nh, nkv, hd, positions, self.cos, self.sin, hd, None, None,
                               cfg.rms_norm_eps, True, None, True, slot_map, self.k_cache[li], self.v_cache[li])
            attn = prefill_attention(qkv[:, : nh * hd], self.k_cache[li], self.v_cache[li], bt, aux["cu"],
                                     kv_lens, aux["tiles"][0], aux["tiles"][1], nh, nkv, hd, causal=True,
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
        idx = (codes.long() + m.code_offset.view(1, -1, 1)).permute(0, 2, 1)
        x = m.code_embedding[idx].float().mean(2).to(cfg.dtype).reshape(B * W, H)
        p0 = torch.zeros(B, dtype=torch.int32, device=x.device) if fresh else self.pos.index_select(0, slots)
        x = self._transformer(x, slots, p0, B, W, aux).view(B, W, H)
        # the sink slot stays at frame 0, however many padding rows pass through it
        self.pos.index_copy_(0, slots, torch.where(slots == self.sink, 0, p0 + W).to(torch.int32))
        ci = 0
        for f, U in zip(cfg.upsampling_ratios, m.up):
            Tc = x.shape[1]
            y = ops.linear(x.contiguous(), U.tconv_w)
            x = (y.view(B, Tc, f, -1) + U.tconv_b).reshape(B, Tc * f, -1).to(cfg.dtype)
            inp = x
            xf = self._history(ci, x, slots, fresh)
            ci += 1
            h = A.dwconv1d_causal(xf, U.dw_w, U.dw_b)[:, xf.shape[1] - x.shape[1]:].contiguous()
            h = ops.layer_norm(h, U.ln_w, U.ln_b, 1e-6)
            h = ops.linear(h, U.pw1_w, bias=U.pw1_b, act="gelu")
            x = ops.linear(h, U.pw2_w, bias=U.pw2_b, residual=inp)
        xf = self._history(ci, x, slots, fresh)
        ci += 1
        x = A.causal_conv1d(xf, m.conv_in_w, m.conv_in_b, 7, pad_left=0, t_out=x.shape[1])
        for r, Bk in zip(cfg.upsample_rates, m.blocks):
            s = A.snake(x, Bk.snake_a, Bk.snake_b)
            if fresh:     # no earlier input: the trimmed output starts at block 0
                self._keep_last(ci, s, slots)
                x = A.conv_transpose1d(s, Bk.tconv_w, Bk.tconv_b, r)
            else:         # the kept sample completes the block the previous chunk held back
                x = A.conv_transpose1d(self._history(ci, s, slots, False), Bk.tconv_w, Bk.tconv_b, r)
            ci += 1
            for Un in Bk.units:
                res = x
                h = A.snake(x, Un.a1, Un.b1)
                hf = self._history(ci, h, slots, fresh)
                ci += 1
                h = A.causal_conv1d(hf, Un.c1_w, Un.c1_b, 7, dilation=Un.dil, pad_left=0, t_out=h.shape[1])
                h = A.snake(h, Un.a2, Un.b2)
                x = A.causal_conv1d(h, Un.c2_w, Un.c2_b, 1, residual=res)
        s = A.snake(x, m.out_snake_a, m.out_snake_b)
        sf = self._history(ci, s, slots, fresh)
        wav = A.causal_conv1d(sf, m.conv_out_w, m.conv_out_b, 7, pad_left=0, t_out=s.shape[1])
        return wav.float().reshape(B, -1).clamp(-1.0, 1.0)


class StatefulGraphs:
    """CUDA graphs of ``Code2WavStreamState.step``, one per (batch bucket, frames, first).

    Padding rows of a bucket decode code 0 through the sink slot.  Graphs are
    captured with the sink in every row, so their warm-up run advances no
    stream's state.  Returned rows view the graph's output buffer: read them
    before the same graph replays."""

    BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128)

    def __init__(self, state: Code2WavStreamState, max_batch: int = 32):
        self.state = state
        self.max_batch = max_batch
        self.graphs: dict[tuple[int, int, bool], tuple] = {}
        self._pool = None

    @torch.no_grad()
    def capture(self, B: int, W: int, fresh: bool) -> None:
        from ...utils.cuda_graph import capture_graph

        st = self.state
        dev = st.pos.device
        codes = torch.zeros(B, st.model.cfg.num_quantizers, W, dtype=torch.long, device=dev)
        slots = torch.full((B,), st.sink, dtype=torch.long, device=dev)
        aux = st.make_aux(B, W)
        with torch.cuda.device(dev):
            g, out = capture_graph(lambda: st.step(codes, slots, fresh, aux), warmup=1, pool=self._pool)
        self._pool = g.pool()
        self.graphs[(B, W, fresh)] = (g, codes, slots, aux, out)

    def capture_all(self, frames: list[tuple[int, bool]]) -> None:
        for W, fresh in frames:
            for B in self.BUCKETS:
                if B > self.max_batch:
                    break
                if (B, W, fresh) not in self.graphs:
                    self.capture(B, W, fresh)

    def bucket(self, B: int) -> int | None:
        return next((b for b in self.BUCKETS if b >= B and b <= self.max_batch), None)

    @torch.no_grad()
    def __call__(self, codes: torch.Tensor, slots: torch.Tensor, fresh: bool) -> torch.Tensor:
        B, _, W = codes.shape
        Bb = self.bucket(B)
        hit = self.graphs.get((Bb, W, fresh)) if Bb is not None else None
        if hit is None:
            return self.state.step(codes, slots, fresh)
        g, cbuf, sbuf, _, out = hit
        cbuf[:B].copy_(codes, non_blocking=True)
        sbuf[:B].copy_(slots, non_blocking=True)
        if B < Bb:
            cbuf[B:].zero_()
            sbuf[B:].fill_(self.state.sink)
        g.replay()
        return out[:B]


@dataclass
class _Stream:
    slot: int
    codes: list = field(default_factory=list)   # [Q] code columns
    emitted_frames: int = 0


class StatefulStreamingCode2Wav:
    """Incremental decoding of many streams with kept state (same interface as
    ``code2wav.StreamingCode2Wav``): every ``chunk`` new frames (or at the end)
    each ready stream decodes only its new frames; ready streams with the same
    (frames, first chunk) run as one batched step.

    Capacity: ``max_streams`` open streams (a slot each, freed by ``close``),
    ``max_frames`` frames per stream."""

    def __init__(self, model: Code2Wav, chunk: int = 10, first_chunk: int | None = None, max_streams: int = 32,
                 max_frames: int = 16384, use_graphs: bool = True):
        self.model = model
        self.chunk = chunk
        self.first_chunk = first_chunk or chunk
        # a step carries one chunk, or what is left of a stream (less than a chunk) at its end
        self.max_step = max(self.chunk, self.first_chunk)
        self.state = Code2WavStreamState(model, max_streams, max_frames, self.max_step)
        dev = model.code_embedding.device
        self.graphs = StatefulGraphs(self.state, max_streams) if use_graphs and dev.type == "cuda" else None
        self.streams: dict[str, _Stream] = {}
        self._free = list(range(max_streams - 1, -1, -1))
        self._pinned: torch.Tensor | None = None

    def step_shapes(self) -> list[tuple[int, bool]]:
        return [(self.first_chunk, True), (self.chunk, False)]

    def capture_graphs(self) -> None:
        if self.graphs is not None:
            self.graphs.capture_all(self.step_shapes())

    def add_codes(self, rid: str, codes: torch.Tensor) -> None:
        """codes: [Q] or [T, Q] frames for stream rid."""
        st = self.streams.get(rid)
        if st is None:
            if not self._free:
                raise RuntimeError(f"code2wav: more than {self.state.S - 1} open streams")
            st = self.streams[rid] = _Stream(self._free.pop())
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

    def _frames(self, st: _Stream, fin: bool) -> int:
        """Frames of the stream's next step: one chunk (the first chunk's size first), or what is
        left at the end (fewer)."""
        pending = len(st.codes) - st.emitted_frames
        need = self.first_chunk if st.emitted_frames == 0 else self.chunk
        return min(need, pending)

    @torch.no_grad()
    def decode_ready(self, rids: list[str], final: bool = False, finals=None,
                     to_host: bool = False) -> dict[str, torch.Tensor]:
        """{rid: float32 waveform of its new frames} for every ready stream (``final`` / ``finals``
        flush the streams whose last frame has arrived).  A stream with several chunks pending
        runs its chunks in successive steps of this call, concatenated.  ``to_host``: numpy
        arrays, copied with one device-to-host transfer per step group."""
        dev = self.model.code_embedding.device
        parts: dict[str, list] = {}
        live = [r for r in rids if r in self.streams]
        fin_of = {r: final or (finals is not None and r in finals) for r in live}
        while True:
            groups: dict[tuple[int, bool], list[tuple[str, torch.Tensor]]] = {}
            for rid in live:
                st = self.streams[rid]
                if not self.ready(rid, fin_of[rid]):
                    continue
                W = self._frames(st, fin_of[rid])
                if st.emitted_frames + W > self.state.max_frames:
                    raise ValueError(f"code2wav stream {rid}: longer than max_frames {self.state.max_frames}")
                fresh = st.emitted_frames == 0
                window = torch.stack(st.codes[st.emitted_frames:st.emitted_frames + W], 1)  # [Q, W]
                groups.setdefault((W, fresh), []).append((rid, window))
                st.emitted_frames += W
            if not groups:
                break
            for (W, fresh), items in groups.items():
                top = self.graphs.max_batch if self.graphs is not None else len(items)
                for i in range(0, len(items), max(1, top)):
                    part = items[i:i + max(1, top)]
                    self._run(part, W, fresh, dev, to_host, parts)
        out = {}
        for rid, ps in parts.items():
            if to_host:
                out[rid] = ps[0] if len(ps) == 1 else np.concatenate(ps)
            else:
                out[rid] = ps[0] if len(ps) == 1 else torch.cat(ps)
        return out

    def _run(self, items, W, fresh, dev, to_host, parts) -> None:
        codes = torch.stack([w for _, w in items], 0).to(dev, non_blocking=True)
        slots = torch.tensor([self.streams[r].slot for r, _ in items], dtype=torch.long).to(dev)
        run = self.graphs if self.graphs is not None else (lambda c, s, f: self.state.step(c, s, f))
        wav = run(codes, slots, fresh)
        if to_host and wav.is_cuda:
            if self._pinned is None or self._pinned.numel() < wav.numel():
                self._pinned = torch.empty(max(wav.numel(), 1 << 20), dtype=torch.float32, pin_memory=True)
            host = self._pinned[:wav.numel()].view(wav.shape)
            host.copy_(wav, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
            for (rid, _), wv in zip(items, host):
                parts.setdefault(rid, []).append(wv.numpy().copy())
        else:
            for (rid, _), wv in zip(items, wav):
                parts.setdefault(rid, []).append(wv.float().cpu().numpy().copy() if to_host else wv.clone())

    def close(self, rid: str) -> None:
        st = self.streams.pop(rid, None)
        if st is not None:
            self._free.append(st.slot)
