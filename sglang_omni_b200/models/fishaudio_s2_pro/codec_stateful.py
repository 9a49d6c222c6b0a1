"""Stateful streaming S2-Pro DAC decoding: every chunk runs only its new code frames.

The DAC decoder (``codec.DACDecoder``) is causal end to end: a window-128
transformer over the code frames, then upsampling, causal convolutions and
causal transposed convolutions (kernel 2s, stride s, left edge kept, so output
block j needs input samples j and j - 1).  This decoder keeps per stream the
transformer's keys / values in a KV ring and every convolution's input history
(``models.common.stream_state``), so the chunks of a stream concatenate to the
full-sequence ``DACDecoder.decode`` of all its frames, each chunk of W frames
giving W * hop samples.

The reference streams by re-decoding every code so far after 5 and then every
100 tokens (sglang_omni/models/fishaudio_s2_pro/pipeline/stages.py:279-280);
the windowed mode of this package's TTS stage re-decodes a 48-frame context
before every chunk.  Here a chunk costs its own frames only.
"""
from __future__ import annotations

import torch

from ... import ops
from ...ops import audio as A
from ...ops.attention import prefill_attention
from ..common.stream_state import ConvHistory, KVRing, SlotStreams, StepGraphs, step_aux
from .codec import DACDecoder


def dac_conv_history(dec: DACDecoder) -> list[tuple[int, int]]:
    """(input samples kept, channels) of every stateful convolution of the decoder, in order."""
    D = dec.cfg.latent_dim
    out = [(U.dw_w.shape[1] - 1, D) for U in dec.up]
    out.append((6, D))                                      # conv_in, kernel 7
    for Bk in dec.blocks:
        out.append((1, Bk.alpha.shape[0]))                  # transposed conv: one input sample
        for Un in Bk.units:
            out.append((6 * Un.dil, Bk.tconv_b.shape[0]))   # kernel 7, dilation dil
    out.append((6, dec.out_alpha.shape[0]))                 # conv_out, kernel 7
    return out


class DACStreamState:
    """Per-slot streaming state of one DAC decoder and the chunk step over it (slot
    ``max_streams`` is the sink of padding rows)."""

    def __init__(self, dec: DACDecoder, max_streams: int, max_frames: int = 8192, max_step: int = 64):
        cfg = dec.cfg
        self.dec = dec
        self.device = dec.rvq_table.device
        self.sink = max_streams
        self.max_frames = max_frames
        self.max_step = max_step
        S = max_streams + 1
        self.kv = KVRing(len(dec.tf), cfg.tf_heads, cfg.tf_head_dim, cfg.tf_window, max_step, S, max_frames,
                         cfg.rope_base, cfg.dtype, self.device, round_bf16=True)
        self.pos = torch.zeros(S, dtype=torch.int32, device=self.device)
        self.hist = ConvHistory(dac_conv_history(dec), S, cfg.dtype, self.device)

    def state_bytes(self) -> int:
        t = self.kv.tensors() + self.hist.t + [self.pos]
        return sum(x.numel() * x.element_size() for x in t)

    def make_aux(self, B: int, W: int) -> dict:
        return step_aux(B, W, 1, self.device)

    def _transformer(self, h: torch.Tensor, slots: torch.Tensor, p0: torch.Tensor, aux: dict) -> torch.Tensor:
        dec, cfg = self.dec, self.dec.cfg
        nh, hd = cfg.tf_heads, cfg.tf_head_dim
        D = nh * hd
        positions, slot_map, kv_lens, bt = self.kv.plan(slots, p0, aux["offs"])
        for li, L in enumerate(dec.tf):
            n1 = ops.rms_norm(h, L.ln1, cfg.norm_eps)
            qkv = ops.linear(n1, L.qkv)
            ops.qkv_rope_store(qkv, nh, nh, hd, positions, self.kv.cos, self.kv.sin, hd, None, None, cfg.norm_eps,
                               False, slot_mapping=slot_map, k_cache=self.kv.k[li], v_cache=self.kv.v[li])
            a = prefill_attention(qkv[:, :D], self.kv.k[li], self.kv.v[li], bt, aux["cu"], kv_lens,
                                  aux["tiles"][0], aux["tiles"][1], nh, nh, hd, causal=True, window=cfg.tf_window)
            h = ops.linear(a, L.o, residual=h)
            n2 = ops.rms_norm(h, L.ln2, cfg.norm_eps)
            h = ops.linear(ops.linear(n2, L.w13, gated=True), L.w2, residual=h)
        return ops.rms_norm(h, dec.tf_norm, cfg.norm_eps)

    @torch.no_grad()
    def step(self, codes: torch.Tensor, slots: torch.Tensor, fresh: bool, aux: dict | None = None) -> torch.Tensor:
        """codes [B, 10, W] and slots [B] (int64) on the decoder's device -> float32 waveform
        rows [B, W * hop] in [-1, 1].  ``fresh``: every row is the first chunk of a new stream
        in its slot.  Advances every slot's state."""
        dec, cfg = self.dec, self.dec.cfg
        B, _, W = codes.shape
        if W > self.max_step:
            raise ValueError(f"DAC step of {W} frames > max_step {self.max_step}")
        aux = aux if aux is not None else self.make_aux(B, W)
        D = cfg.latent_dim
        hist = self.hist
        p0 = torch.zeros(B, dtype=torch.int32, device=codes.device) if fresh else self.pos.index_select(0, slots)
        x = self._transformer(dec._rvq(codes), slots, p0, aux).view(B, W, D)
        # the sink slot stays at frame 0, however many padding rows pass through it
        self.pos.index_copy_(0, slots, torch.where(slots == self.sink, 0, p0 + W).to(torch.int32))
        ci = 0
        for U in dec.up:
            Tc = x.shape[1]
            y = ops.linear(x.reshape(B * Tc, D), U.tconv_w, out_dtype=torch.float32)
            x = (y.view(B, Tc, U.f, D) + U.tconv_b.float()).reshape(B, Tc * U.f, D).to(cfg.dtype)
            inp = x
            xf = hist.extend(ci, x, slots, fresh)
            ci += 1
            h = A.dwconv1d_causal(xf, U.dw_w, U.dw_b)[:, xf.shape[1] - x.shape[1]:].contiguous()
            h = ops.layer_norm(h, U.ln_w, U.ln_b, 1e-6)
            h = ops.linear(h, U.pw1_w, bias=U.pw1_b, act="gelu")
            x = ops.linear(h, U.pw2_w, bias=U.pw2_b, residual=inp)
        xf = hist.extend(ci, x, slots, fresh)
        ci += 1
        x = A.causal_conv1d(xf, dec.conv_in_w, dec.conv_in_b, 7, pad_left=0, t_out=x.shape[1])
        for Bk in dec.blocks:
            s = A.snake(x, Bk.alpha, None, log_scale=False)
            Tn = s.shape[1]
            # the kept input sample (zero for a new stream) supplies the overlap of block 0
            sf = hist.extend(ci, s, slots, fresh)
            ci += 1
            x = A.conv_transpose1d(sf, Bk.tconv_w, Bk.tconv_b, Bk.stride, trim_left=Bk.stride, t_out=Tn * Bk.stride)
            for Un in Bk.units:
                h = A.snake(x, Un.a1, None, log_scale=False)
                hf = hist.extend(ci, h, slots, fresh)
                ci += 1
                h = A.causal_conv1d(hf, Un.c1_w, Un.c1_b, 7, dilation=Un.dil, pad_left=0, t_out=h.shape[1])
                h = A.snake(h, Un.a2, None, log_scale=False)
                x = A.causal_conv1d(h, Un.c2_w, Un.c2_b, 1, residual=x)
        s = A.snake(x, dec.out_alpha, None, log_scale=False)
        sf = hist.extend(ci, s, slots, fresh)
        wav = A.causal_conv1d(sf, dec.conv_out_w, dec.conv_out_b, 7, pad_left=0, t_out=s.shape[1])
        return torch.tanh(wav.float().reshape(B, -1))


class StatefulStreamingDAC(SlotStreams):
    """Incremental DAC decoding of many S2-Pro streams with kept state: the first
    ``first_chunk`` frames, then every ``chunk`` new frames (or what is left at the end),
    each ready stream decodes only its new frames, batched with the others.  Codes are
    [10] columns per frame (semantic code, then the 9 residual codes)."""

    def __init__(self, dec: DACDecoder, chunk: int = 20, first_chunk: int | None = None, max_streams: int = 64,
                 max_frames: int = 8192, use_graphs: bool = True, max_batch: int = 64):
        state = DACStreamState(dec, max_streams, max_frames, max(chunk, first_chunk or chunk))
        graphs = (StepGraphs(state, dec.cfg.num_codebooks, min(max_batch, max_streams))
                  if use_graphs and state.device.type == "cuda" else None)
        super().__init__(state, chunk, first_chunk, graphs)
        self.dec = dec
