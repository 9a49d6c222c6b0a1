"""Batched dual-AR decoding for S2-Pro: every active stream advances one frame
per step, and the whole step is one CUDA-graph replay per batch bucket.

One frame (reference: S2ProSGLangTextModel.forward + _decode_codebooks,
sglang_omni/models/fishaudio_s2_pro/sglang_model.py:290-377, and the runner's
VQ buffer updates, runtime/s2pro_sglang_ar.py:377-470):

  1. input row of every stream = E[previous token], plus at semantic tokens the
     sum of the previous frame's 10 codebook embeddings, times 1/sqrt(11)
     (``ops.vq_embed``, reading per-slot device state);
  2. slow AR decode over the paged KV cache;
  3. constrained semantic sampling over the 4096 semantic rows + <|im_end|>
     of the tied LM head;
  4. fast AR: position 0 = project_in(hidden), then the semantic code and
     codebooks 1..9 one position at a time (one 64-slot KV page per stream),
     each sampled from the 4096-way codebook head;
  5. the frame's codes go to per-slot device state (next step's input) and to
     the output rows [token, code_0 .. code_9].

Per-request sampling state lives in slot-indexed device arrays, so the graph
replays for any mix of requests.  Prefill runs eagerly (ragged prompts with
VQ parts) and ends with the same steps 3-5.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from ... import ops
from ...engines.ar.kv_pool import KVPool
from ...environ import environ
from ...ops.sampling import SamplingTensors, sample
from ...utils.cuda_graph import capture_graph
from ...utils.hostdev import h2d
from ...utils.staging import PinnedRing
from ..decoder import ForwardBatch
from .model import S2ProDualAR


@dataclass
class TTSStream:
    rid: str
    slot: int
    prompt_ids: list
    code_rows: torch.Tensor                 # int32 [len(prompt)] row of vq_codes or -1
    vq_codes: torch.Tensor                  # int32 [n_vq, num_codebooks]
    max_new_tokens: int = 1024
    pages: list = field(default_factory=list)
    num_cached: int = 0
    frames: int = 0
    finished: bool = False
    prefilled: bool = False


class DualARGenerator:
    def __init__(self, model: S2ProDualAR, max_streams: int = 64, max_context: int = 4096,
                 use_graphs: bool = True, max_prefill_tokens: int = 8192):
        self.model = model
        cfg = model.cfg
        sc, fc = cfg.slow, cfg.fast
        dev = model.slow.embed.device
        self.device = dev
        self.cfg = cfg
        self.ncb = cfg.num_codebooks
        self.max_streams = max_streams
        self.max_pages = (max_context + 63) // 64
        self.max_prefill_tokens = max_prefill_tokens
        self.pool = KVPool(sc.num_layers, sc.num_kv_heads, sc.head_dim, max_streams * self.max_pages + 2, dev, sc.dtype)
        # one fast-AR page per slot (num_codebooks positions <= 64)
        self.fast_pool = KVPool(fc.num_layers, fc.num_kv_heads, fc.head_dim, max_streams + 2, dev, fc.dtype)
        model.slow.ensure_workspaces(max_prefill_tokens, max_streams, max_context)
        model.fast.ensure_workspaces(max_streams, max_streams, 64)
        S = max_streams + 1  # slot 0 = padding rows of a bucket
        self.S = S
        self.slot_tokens = torch.zeros(S, dtype=torch.int32, device=dev)
        self.prev_codes = torch.zeros(S, self.ncb, dtype=torch.int32, device=dev)
        self.out_codes = torch.zeros(S, self.ncb + 1, dtype=torch.int32, device=dev)
        self.sem_idx_tok = torch.zeros(S, dtype=torch.int32, device=dev)
        self.cb_tok = torch.zeros(S, dtype=torch.int32, device=dev)
        V = cfg.codebook_size + 1
        self.sem_st = SamplingTensors(torch.zeros(S, device=dev), torch.zeros(S, dtype=torch.int32, device=dev),
                                      torch.ones(S, device=dev), torch.zeros(S, device=dev), torch.ones(S, device=dev),
                                      torch.zeros(S, V, dtype=torch.uint8, device=dev),
                                      torch.arange(S, dtype=torch.int64, device=dev) * 7919,
                                      torch.zeros(S, dtype=torch.int32, device=dev))
        self.cb_st = SamplingTensors(torch.zeros(S, device=dev), torch.zeros(S, dtype=torch.int32, device=dev),
                                     torch.ones(S, device=dev), None, None, None,
                                     torch.arange(S, dtype=torch.int64, device=dev) * 104729,
                                     torch.zeros(S, dtype=torch.int32, device=dev))
        self.streams: dict[str, TTSStream] = {}
        self.free_slots = list(range(S - 1, 0, -1))
        self.use_graphs = use_graphs and dev.type == "cuda" and environ.OMNI_USE_CUDA_GRAPHS.get()
        self.graphs: dict[int, tuple] = {}
        self.buckets = [b for b in (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128) if b <= max_streams]
        if self.buckets[-1] < max_streams:
            self.buckets.append(max_streams)
        PB = max_streams
        self.meta_ring = PinnedRing(6 * PB + PB * self.max_pages, torch.int32, 2, dev.type == "cuda")
        self.meta_dev = torch.zeros(6 * PB + PB * self.max_pages, dtype=torch.int32, device=dev)
        try:
            from ... import _runtime as rt
            self.builder = rt.DecodeMetaBuilder(PB, self.max_pages)
        except ImportError:  # pragma: no cover
            self.builder = None

    # ------------------------------------------------------------------ streams
    def add_stream(self, rid: str, prompt_ids: list, code_rows: torch.Tensor, vq_codes: torch.Tensor,
                   max_new_tokens: int = 1024, temperature: float = 0.8, top_p: float = 0.8, top_k: int = 30,
                   repetition_penalty: float = 1.1, seed: int | None = None) -> TTSStream:
        if not self.free_slots:
            raise RuntimeError("no free stream slot")
        slot = self.free_slots.pop()
        cap = self.max_pages * 64 - len(prompt_ids)
        if cap < 1:
            self.free_slots.append(slot)
            raise ValueError(f"prompt of {len(prompt_ids)} tokens exceeds the context of {self.max_pages * 64}")
        st = TTSStream(rid, slot, list(prompt_ids), code_rows, vq_codes, max(1, min(max_new_tokens, cap)))
        self.streams[rid] = st
        t = float(temperature)
        self.sem_st.temperature[slot] = t
        self.sem_st.top_k[slot] = int(top_k)
        self.sem_st.top_p[slot] = float(top_p)
        self.sem_st.rep_penalty[slot] = float(repetition_penalty)
        self.sem_st.seen[slot].zero_()
        self.sem_st.step[slot] = 0
        self.cb_st.temperature[slot] = t
        self.cb_st.top_k[slot] = int(top_k)
        self.cb_st.top_p[slot] = float(top_p)
        self.cb_st.step[slot] = 0
        if seed is not None:
            m = (1 << 62) - 1
            self.sem_st.seeds[slot] = int(seed) & m
            self.cb_st.seeds[slot] = (int(seed) * 31 + 7) & m
        return st

    def remove(self, rid: str) -> None:
        st = self.streams.pop(rid, None)
        if st is not None:
            self.pool.free(st.pages)
            self.free_slots.append(st.slot)

    def active(self) -> list[TTSStream]:
        return [s for s in self.streams.values() if s.prefilled and not s.finished]

    # ------------------------------------------------------------------ frame tail (steps 3-5)
    def _tail(self, hidden: torch.Tensor, slots: torch.Tensor) -> torch.Tensor:
        m, cfg = self.model, self.cfg
        B = hidden.shape[0]
        dev = hidden.device
        logits = ops.linear(hidden, m.sem_head, out_dtype=torch.float32)
        idx = sample(logits, self.sem_st, row_slot=slots, slot_tokens=self.sem_idx_tok)
        is_end = idx >= cfg.codebook_size
        token = torch.where(is_end, torch.full_like(idx, cfg.im_end_id), idx + cfg.semantic_begin_id)
        sem_code = torch.where(is_end, torch.zeros_like(idx), idx)
        # fast AR over this frame
        fast = m.fast
        x = ops.linear(hidden, m.project_in_w, bias=m.project_in_b) if m.has_project_in else hidden
        bt = (slots + 1).view(-1, 1).to(torch.int32)
        base = (slots + 1) * 64
        codes = [sem_code]
        code = sem_code
        for j in range(self.ncb):
            pos = torch.full((B,), j, dtype=torch.int32, device=dev)
            fb = ForwardBatch(is_decode=True, positions=pos, slot_mapping=base + j,
                              kv_lens=torch.full((B,), j + 1, dtype=torch.int32, device=dev), block_table=bt,
                              input_embeds=x)
            h = fast(fb, self.fast_pool.kv)
            if j == 0:
                x = fast.embed[sem_code.long()]
                continue
            lg = ops.linear(h, fast.head_weight, out_dtype=torch.float32)
            code = sample(lg, self.cb_st, row_slot=slots, slot_tokens=self.cb_tok)
            codes.append(code)
            if j + 1 < self.ncb:
                x = fast.embed[code.long()]
        frame = torch.stack(codes, 1)                      # [B, ncb]
        sl = slots.long()
        self.prev_codes[sl] = frame
        self.slot_tokens[sl] = token
        out = torch.cat([token.view(-1, 1), frame], 1)
        self.out_codes[sl] = out
        return out

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, streams: list[TTSStream]) -> torch.Tensor:
        """Runs the prompts of ``streams`` (one ragged batch) and their first frame; returns codes [B, ncb+1]."""
        m, cfg, dev = self.model, self.cfg, self.device
        sl = m.slow
        lens = [len(s.prompt_ids) for s in streams]
        for s, n in zip(streams, lens):
            need = KVPool.pages_for(n) - len(s.pages)
            if need > 0:
                s.pages.extend(self.pool.alloc(need))
        cu = np.zeros(len(streams) + 1, dtype=np.int32)
        cu[1:] = np.cumsum(lens)
        pos = np.concatenate([np.arange(n, dtype=np.int32) for n in lens])
        slot_map = np.concatenate([np.asarray(s.pages)[np.arange(n) // 64] * 64 + np.arange(n) % 64
                                   for s, n in zip(streams, lens)]).astype(np.int32)
        bt = np.zeros((len(streams), max(len(s.pages) for s in streams)), dtype=np.int32)
        for i, s in enumerate(streams):
            bt[i, :len(s.pages)] = s.pages
        ids = np.concatenate([np.asarray(s.prompt_ids, dtype=np.int32) for s in streams])
        rows, codes, base = [], [], 0
        for s in streams:
            r = s.code_rows.to(torch.int32).clone()
            r[r >= 0] += base
            rows.append(r)
            codes.append(s.vq_codes.to(torch.int32).reshape(-1, self.ncb))
            base += s.vq_codes.shape[0]
        code_rows = torch.cat(rows)
        all_codes = torch.cat(codes, 0) if base else torch.zeros(1, self.ncb, dtype=torch.int32)
        d = lambda a: h2d(a, dev)  # noqa: E731
        x = ops.vq_embed(sl.embed, m.codebook_embeddings, d(all_codes), cfg.codebook_size, cfg.vq_scale,
                         cfg.semantic_begin_id, cfg.semantic_end_id, ids=d(ids), code_row=d(code_rows))
        G = sl.cfg.num_heads // sl.cfg.num_kv_heads
        rows = ops.prefill_tile_rows(sl.cfg.head_dim, G) if dev.type == "cuda" else 64
        req, tok0 = ops.prefill_tiles(lens, G, rows)
        fb = ForwardBatch(is_decode=False, positions=d(pos), slot_mapping=d(slot_map),
                          kv_lens=h2d(lens, dev, torch.int32), block_table=d(bt),
                          input_embeds=x, cu_q=d(cu), tile_req=h2d(req, dev, torch.int32),
                          tile_tok0=h2d(tok0, dev, torch.int32), tile_rows=rows, logits_indices=d(cu[1:] - 1))
        hidden = sl(fb, self.pool.kv)
        slots = h2d([s.slot for s in streams], dev, torch.int32)
        out = self._tail(hidden, slots)
        for s, n in zip(streams, lens):
            s.num_cached = n
            s.frames = 1
            s.prefilled = True
        return out

    # ------------------------------------------------------------------ decode
    def _bucket(self, n: int) -> int:
        for b in self.buckets:
            if b >= n:
                return b
        raise ValueError(n)

    def _views(self, PB: int):
        mt = self.meta_dev
        P = self.max_pages
        return (mt[0:PB], mt[PB:2 * PB], mt[2 * PB:3 * PB], mt[5 * PB:6 * PB],
                mt[6 * PB:6 * PB + PB * P].view(PB, P))

    def _step_body(self, PB: int) -> torch.Tensor:
        m, cfg = self.model, self.cfg
        kv_lens, slot_mapping, positions, slots, bt = self._views(PB)
        x = ops.vq_embed(m.slow.embed, m.codebook_embeddings, self.prev_codes, cfg.codebook_size, cfg.vq_scale,
                         cfg.semantic_begin_id, cfg.semantic_end_id, slot=slots, slot_tokens=self.slot_tokens)
        fb = ForwardBatch(is_decode=True, positions=positions, slot_mapping=slot_mapping, kv_lens=kv_lens,
                          block_table=bt, input_embeds=x)
        hidden = m.slow(fb, self.pool.kv)
        return self._tail(hidden, slots)

    def _fill_meta(self, streams: list[TTSStream], PB: int):
        host = self.meta_ring.next().numpy()
        B = len(streams)
        kl = np.fromiter((s.num_cached for s in streams), dtype=np.int64, count=B)
        md = np.zeros(B, dtype=np.int64)
        sl = np.fromiter((s.slot for s in streams), dtype=np.int64, count=B)
        if self.builder is not None:
            self.builder.build(host, [s.pages for s in streams], kl, md, sl, self.pool.allocator_native(), PB)
        else:  # same packed layout as the native builder
            P = self.max_pages
            for s, k in zip(streams, kl):
                if int(k) // 64 >= len(s.pages):
                    s.pages.extend(self.pool.alloc(1))
            host[:6 * PB + PB * P] = 0
            host[0:B] = kl + 1
            host[PB:PB + B] = [s.pages[int(k) // 64] * 64 + int(k) % 64 for s, k in zip(streams, kl)]
            host[PB + B:2 * PB] = -1
            for j in range(3):
                host[(2 + j) * PB:(2 + j) * PB + B] = kl
            host[5 * PB:5 * PB + B] = sl
            for i, s in enumerate(streams):
                host[6 * PB + i * P:6 * PB + i * P + len(s.pages)] = s.pages
        n = 6 * PB + PB * self.max_pages
        self.meta_ring.upload(self.meta_dev, n)

    def capture_all(self):
        """Captures the frame-step graph of every batch bucket up front."""
        if self.use_graphs:
            for PB in self.buckets:
                if PB not in self.graphs:
                    self._capture(PB)

    def _capture(self, PB: int):
        host = self.meta_ring.next().numpy()
        n = 6 * PB + PB * self.max_pages
        host[:n] = 0
        host[PB:2 * PB] = -1
        self.meta_ring.upload(self.meta_dev, n, blocking=True)
        saved = [t.clone() for t in (self.prev_codes, self.slot_tokens, self.out_codes, self.sem_st.step,
                                     self.cb_st.step, self.sem_st.seen[0])]
        self.graphs[PB] = capture_graph(lambda: self._step_body(PB))
        # padding rows only touched slot 0; put back what the warm-up changed
        for dst, src in zip((self.prev_codes, self.slot_tokens, self.out_codes, self.sem_st.step, self.cb_st.step,
                             self.sem_st.seen[0]), saved):
            dst.copy_(src)

    @torch.no_grad()
    def step(self, streams: list[TTSStream]) -> torch.Tensor:
        """One frame for every stream; returns codes [B, ncb+1] (device)."""
        B = len(streams)
        PB = self._bucket(B)
        if self.use_graphs and PB not in self.graphs:
            self._capture(PB)
        self._fill_meta(streams, PB)
        if self.use_graphs:
            g, out = self.graphs[PB]
            g.replay()
        else:
            out = self._step_body(PB)
        for s in streams:
            s.num_cached += 1
            s.frames += 1
        return out[:B]

    def __len__(self):
        return len(self.streams)


def stream_seed(rid: str) -> int:
    """Deterministic per-request seed from the request id."""
    h = 1469598103934665603
    for ch in rid.encode():
        h = ((h ^ ch) * 1099511628211) & ((1 << 63) - 1)
    return h

