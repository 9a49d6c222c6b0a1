"""Per-stream state of streaming vocoders whose chunks run only their new frames.

A streaming vocoder built from a causal sliding-window transformer and causal
convolutions (Qwen3-Omni Code2Wav, the S2-Pro DAC decoder) can decode a stream
chunk by chunk and still produce exactly the waveform of one full-sequence
forward, if each chunk sees what the full forward would have shown it of the
past:

* ``KVRing``: the transformer's keys / values (after RoPE) of each stream and
  layer, in a ring of 64-key pages.  Row ``s`` of the block table maps logical
  page i of stream slot s to physical page ``s * ring + i % ring``; the paged
  prefill attention kernel, given the window, never reads a page wholly below
  a query tile's first visible key, so older pages are overwritten safely.
  Positions are the stream's absolute frame indices.
* ``ConvHistory``: for each causal convolution the last (K - 1) * dilation
  input samples of each stream (one input sample for a transposed convolution
  of kernel 2s / stride s), prepended to the chunk's input.

Streams own slots 0 .. max_streams - 1; slot ``max_streams`` is a sink for the
padding rows of a batch bucket.  Every per-stream tensor is indexed by slot id
on the device, so one step has fixed shapes for a given (batch, frames, first
chunk) and replays as one CUDA graph (``StepGraphs``).  ``SlotStreams`` is the
host-side bookkeeping: frames per stream, chunk schedule, slot allocation and
batching of ready streams into steps.

The reference re-runs a window of earlier frames before every chunk instead
(sglang_omni/models/qwen3_omni/components/code2wav_executor.py:211-232 with 25
context frames; sglang_omni/models/fishaudio_s2_pro/pipeline/stages.py:279-280
re-decodes every code so far).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable

import numpy as np
import torch

from ... import ops
from ...ops.attention import PAGE, prefill_tiles


class KVRing:
    """Paged keys / values of ``layers`` attention layers for ``slots`` streams, kept for a
    causal ``window`` of frames; steps of at most ``max_step`` frames."""

    def __init__(self, layers: int, kv_heads: int, head_dim: int, window: int, max_step: int, slots: int,
                 max_frames: int, rope_theta: float, dtype: torch.dtype, device, round_bf16: bool = True):
        self.window = window
        # keys one step can need: window - 1 before its first frame, plus its own frames
        self.ring = -(-(window - 1 + max_step) // PAGE) + 1
        shape = (slots * self.ring, kv_heads, PAGE, head_dim)
        self.k = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(layers)]
        self.v = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(layers)]
        nbt = -(-max_frames // PAGE)
        s = torch.arange(slots, device=device)[:, None]
        self.block_table = (s * self.ring + torch.arange(nbt, device=device)[None] % self.ring).to(torch.int32)
        self.cos, self.sin = ops.rope_tables(head_dim, rope_theta, max_frames, device, round_bf16=round_bf16)

    def plan(self, slots: torch.Tensor, p0: torch.Tensor, offs: torch.Tensor):
        """(positions [B*W] int32, KV slot of each new frame [B*W] int32, keys visible [B] int32,
        block-table rows [B, pages]) of a step whose streams start at frame ``p0``."""
        B, W = slots.shape[0], offs.shape[0]
        pos2 = p0.view(B, 1) + offs.view(1, W)
        page = slots.view(B, 1) * self.ring + torch.div(pos2, PAGE, rounding_mode="floor") % self.ring
        slot_map = (page * PAGE + pos2 % PAGE).reshape(-1).to(torch.int32)
        return (pos2.reshape(-1), slot_map, (p0 + W).to(torch.int32),
                self.block_table.index_select(0, slots))

    def tensors(self) -> list[torch.Tensor]:
        return self.k + self.v + [self.block_table, self.cos, self.sin]


class ConvHistory:
    """The kept input samples of every stateful convolution, per slot: ``shapes`` lists
    (samples kept, channels) in forward order."""

    def __init__(self, shapes: list[tuple[int, int]], slots: int, dtype: torch.dtype, device):
        self.t = [torch.zeros(slots, n, c, dtype=dtype, device=device) for n, c in shapes]

    def extend(self, i: int, x: torch.Tensor, slots: torch.Tensor, fresh: bool) -> torch.Tensor:
        """[kept samples of conv i; x] per stream ([B, n + T, C]), and the new kept samples
        stored.  A stream's first chunk (``fresh``) starts from zeros, the causal padding."""
        st = self.t[i]
        n = st.shape[1]
        prev = x.new_zeros(x.shape[0], n, x.shape[2]) if fresh else st.index_select(0, slots)
        xf = torch.cat([prev, x], 1)
        st.index_copy_(0, slots, xf[:, xf.shape[1] - n:])
        return xf

    def keep_last(self, i: int, x: torch.Tensor, slots: torch.Tensor) -> None:
        st = self.t[i]
        st.index_copy_(0, slots, x[:, x.shape[1] - st.shape[1]:])


def step_aux(B: int, W: int, group: int, device) -> dict:
    """Device tensors of a [B streams, W frames] step that depend only on its shape."""
    req, tok0 = prefill_tiles([W] * B, group, 64)
    return {"offs": torch.arange(W, dtype=torch.int32, device=device),
            "cu": torch.arange(0, (B + 1) * W, W, dtype=torch.int32, device=device),
            "tiles": (torch.tensor(req, dtype=torch.int32, device=device),
                      torch.tensor(tok0, dtype=torch.int32, device=device))}


class StepGraphs:
    """CUDA graphs of ``state.step(codes [B, Q, W], slots [B], fresh, aux)``, one per (batch
    bucket, frames, first chunk).

    Padding rows of a bucket decode code 0 through the sink slot.  Graphs are captured with
    the sink in every row, so their warm-up run advances no stream's state.  Returned rows
    view the graph's output buffer: read them before the same graph replays."""

    BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128)

    def __init__(self, state, code_rows: int, max_batch: int = 32):
        self.state = state
        self.code_rows = code_rows
        self.max_batch = max_batch
        self.graphs: dict[tuple[int, int, bool], tuple] = {}
        self._pool = None

    @torch.no_grad()
    def capture(self, B: int, W: int, fresh: bool) -> None:
        from ...utils.cuda_graph import capture_graph

        st = self.state
        dev = st.device
        codes = torch.zeros(B, self.code_rows, W, dtype=torch.long, device=dev)
        slots = torch.full((B,), st.sink, dtype=torch.long, device=dev)
        aux = st.make_aux(B, W)
        with torch.cuda.device(dev):
            g, out = capture_graph(lambda: st.step(codes, slots, fresh, aux), warmup=1, pool=self._pool)
        self._pool = g.pool()
        self.graphs[(B, W, fresh)] = (g, codes, slots, aux, out)

    def capture_all(self, shapes: list[tuple[int, bool]]) -> None:
        for W, fresh in shapes:
            for B in self.BUCKETS:
                if B > self.max_batch:
                    break
                if (B, W, fresh) not in self.graphs:
                    self.capture(B, W, fresh)

    def bucket(self, B: int) -> int | None:
        return next((b for b in self.BUCKETS if B <= b <= self.max_batch), None)

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
    codes: list = field(default_factory=list)   # one [Q] code column per frame
    emitted_frames: int = 0


class SlotStreams:
    """Incremental decoding of many streams over a stateful decoder ``state`` (``step``,
    ``sink``, ``max_frames``, ``device``): the first ``first_chunk`` frames of a stream, then
    every ``chunk`` new frames (or what is left at the end), each ready stream decodes only
    its new frames; ready streams with the same (frames, first chunk) run as one batched step.

    Capacity: ``state.sink`` open streams (a slot each, freed by ``close``), ``max_frames``
    frames per stream."""

    def __init__(self, state, chunk: int, first_chunk: int | None, graphs: StepGraphs | None):
        self.state = state
        self.chunk = chunk
        self.first_chunk = first_chunk or chunk
        self.graphs = graphs
        self.streams: dict[str, _Stream] = {}
        self._free = list(range(state.sink - 1, -1, -1))
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
                raise RuntimeError(f"streaming decoder: more than {self.state.sink} open streams")
            st = self.streams[rid] = _Stream(self._free.pop())
        if codes.dim() == 1:
            codes = codes.unsqueeze(0)
        st.codes.extend(list(codes))

    def frames(self, rid: str) -> int:
        st = self.streams.get(rid)
        return len(st.codes) if st is not None else 0

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
        """{rid: float32 waveform of its new frames} for every ready stream (``final`` /
        ``finals`` flush the streams whose last frame has arrived).  A stream with several
        chunks pending runs them in successive steps of this call, concatenated.  ``to_host``:
        numpy arrays, copied with one device-to-host transfer per step group."""
        dev = self.state.device
        parts: dict[str, list] = {}
        live = [r for r in rids if r in self.streams]
        fin = {r: final or (finals is not None and r in finals) for r in live}
        while True:
            groups: dict[tuple[int, bool], list[tuple[str, torch.Tensor]]] = {}
            for rid in live:
                st = self.streams[rid]
                if not self.ready(rid, fin[rid]):
                    continue
                need = self.first_chunk if st.emitted_frames == 0 else self.chunk
                W = min(need, len(st.codes) - st.emitted_frames)
                if st.emitted_frames + W > self.state.max_frames:
                    raise ValueError(f"stream {rid}: longer than max_frames {self.state.max_frames}")
                window = torch.stack(st.codes[st.emitted_frames:st.emitted_frames + W], 1)  # [Q, W]
                groups.setdefault((W, st.emitted_frames == 0), []).append((rid, window))
                st.emitted_frames += W
            if not groups:
                break
            for (W, fresh), items in groups.items():
                top = max(1, self.graphs.max_batch if self.graphs is not None else len(items))
                for i in range(0, len(items), top):
                    self._run(items[i:i + top], fresh, dev, to_host, parts)
        out = {}
        for rid, ps in parts.items():
            if len(ps) == 1:
                out[rid] = ps[0]
            else:
                out[rid] = np.concatenate(ps) if to_host else torch.cat(ps)
        return out

    def _run(self, items, fresh: bool, dev, to_host: bool, parts: dict) -> None:
        codes = torch.stack([w for _, w in items], 0).to(dev, non_blocking=True)
        slots = torch.tensor([self.streams[r].slot for r, _ in items], dtype=torch.long).to(dev)
        run: Callable = self.graphs if self.graphs is not None else self.state.step
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
