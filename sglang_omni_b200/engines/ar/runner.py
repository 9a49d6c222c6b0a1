"""Model runner of the paged AR engine: batch metadata -> device, forward,
logits, fused sampling; decode steps replay CUDA graphs captured per batch
bucket.

Per-request state that the device needs every step lives in fixed per-slot
arrays (last token, sampling parameters, RNG step, seen-token mask), so a
decode step reads its input tokens and writes its sampled tokens on the
device, and the host can run one step behind (overlap scheduling).

Reference counterparts: SGLangModelRunner.execute / _forward_with_omni_embeds
(sglang_omni/engines/omni/runtime/sglang_ar.py:501-1046) over SGLang's
ModelRunner + ForwardBatch (sglang_omni/engines/ar/sglang_backend/model_worker.py).
"""
from __future__ import annotations

import zlib

import numpy as np
import torch

from ...models.decoder import DecoderLM, ForwardBatch
from ...ops import prefill_tile_rows, prefill_tiles
from ...ops.sampling import SamplingTensors, sample
from ...environ import environ
from ...utils.cuda_graph import capture_graph
from ...utils.hostdev import adopt, h2d
from ...utils.staging import PinnedRing
from .kv_pool import KVPool
from .request import ARRequest

try:  # native metadata builder (falls back to numpy)
    from ... import _runtime as _rt
except ImportError:  # pragma: no cover
    _rt = None

DEFAULT_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 40, 48, 56, 64, 80, 96, 112, 128, 160, 192, 224, 256)


class ARModelRunner:
    def __init__(self, model: DecoderLM, pool: KVPool, max_batch: int = 64, max_slots: int = 256,
                 max_context: int = 8192, max_prefill_tokens: int = 8192, use_graphs: bool = True,
                 suppress=(-1, -1, -1), track_seen: bool = False, graph_buckets=DEFAULT_BUCKETS):
        self.model = model
        self.pool = pool
        self.device = pool.device
        self.cfg = model.cfg
        self.max_batch = max_batch
        self.max_slots = max_slots
        self.max_pages = (max_context + 63) // 64
        self.max_context = self.max_pages * 64
        self.suppress = suppress
        dev = self.device
        self.is_cuda = dev.type == "cuda"
        model.ensure_workspaces(max(max_prefill_tokens, max_batch), max_batch, self.max_context)
        # per-slot device state
        self.slot_tokens = torch.zeros(max_slots, dtype=torch.int32, device=dev)
        self.temperature = torch.zeros(max_slots, dtype=torch.float32, device=dev)
        self.top_k = torch.zeros(max_slots, dtype=torch.int32, device=dev)
        self.top_p = torch.ones(max_slots, dtype=torch.float32, device=dev)
        self.min_p = torch.zeros(max_slots, dtype=torch.float32, device=dev)
        self.rep = torch.ones(max_slots, dtype=torch.float32, device=dev)
        self.seeds = torch.zeros(max_slots, dtype=torch.int64, device=dev)
        self.step_ctr = torch.zeros(max_slots, dtype=torch.int32, device=dev)
        self.seen = (torch.zeros(max_slots, self.cfg.vocab_size, dtype=torch.uint8, device=dev)
                     if track_seen else None)
        self.st = SamplingTensors(self.temperature, self.top_k, self.top_p, self.min_p,
                                  self.rep if track_seen else None, self.seen, self.seeds, self.step_ctr)
        self.free_slots = list(range(max_slots - 1, 0, -1))  # slot 0 is the padding dummy
        # decode buffers
        self.buckets = [b for b in graph_buckets if b <= max_batch]
        if not self.buckets or self.buckets[-1] < max_batch:
            self.buckets.append(max_batch)
        packed = 6 * max_batch + max_batch * self.max_pages
        self.meta_ring = PinnedRing(packed, torch.int32, 2, self.is_cuda)
        self.meta_dev = torch.zeros(packed, dtype=torch.int32, device=dev)
        # two pinned token buffers: with overlap scheduling step N+1 is launched before step N is read
        self._tok_host = [torch.zeros(max(max_batch, 1024), dtype=torch.int32, pin_memory=self.is_cuda)
                          for _ in range(2)]
        self._tok_flip = 0
        self.builder = _rt.DecodeMetaBuilder(max_batch, self.max_pages) if _rt is not None else None
        self.use_graphs = use_graphs and self.is_cuda and environ.OMNI_USE_CUDA_GRAPHS.get()
        self.graphs: dict[int, tuple] = {}
        self.capture_hidden = False
        self.hidden_out: dict[int, torch.Tensor] = {}

    def _next_tok_host(self) -> torch.Tensor:
        self._tok_flip ^= 1
        return self._tok_host[self._tok_flip]

    # ------------------------------------------------------------------ slots
    def assign_slot(self, req: ARRequest):
        if not self.free_slots:
            raise RuntimeError("no free request slots")
        req.slot = self.free_slots.pop()
        sp = req.sampling
        s = req.slot
        self.temperature[s] = float(sp.temperature) if sp.top_k != 1 else 0.0
        self.top_k[s] = int(sp.top_k) if sp.top_k and sp.top_k > 0 else 0
        self.top_p[s] = float(sp.top_p)
        self.min_p[s] = float(sp.min_p)
        self.rep[s] = float(sp.repetition_penalty)
        # a stable function of the request id (str hash is salted per process): the ranks of a
        # tensor-parallel group draw the same samples
        self.seeds[s] = int(sp.seed if sp.seed is not None else zlib.crc32(req.rid.encode()) & 0x7FFFFFFF)
        self.step_ctr[s] = 0
        if self.seen is not None:
            self.seen[s].zero_()
            if req.prompt_ids and sp.repetition_penalty != 1.0:
                ids = [i for i in req.prompt_ids if 0 <= i < self.cfg.vocab_size]
                self.seen[s, h2d(ids, self.device, torch.long)] = 1

    def release_slot(self, req: ARRequest):
        if req.slot > 0:
            self.free_slots.append(req.slot)
            req.slot = -1

    # ------------------------------------------------------------------ prefill
    def _pos_rows(self, req: ARRequest, start: int, end: int) -> np.ndarray:
        if req.mrope_positions is not None:
            n = req.mrope_positions.shape[1]
            head = req.mrope_positions[:, start:min(end, n)].cpu().numpy().astype(np.int32)
            if end <= n:
                return head
            p = np.arange(max(start, n), end, dtype=np.int32) + req.mrope_delta
            return np.concatenate([head, np.stack([p, p, p])], axis=1)
        p = np.arange(start, end, dtype=np.int32)
        return np.stack([p, p, p])

    @torch.no_grad()
    def prefill(self, chunks: list[tuple[ARRequest, int, int]]):
        """chunks: (request, first prompt token, end token). Returns (sample_rows, event) or None."""
        dev = self.device
        B = len(chunks)
        q_lens = [e - s for _, s, e in chunks]
        T = sum(q_lens)
        ids = np.empty(T, dtype=np.int32)
        pos = np.empty((3, T), dtype=np.int32)
        slots = np.empty(T, dtype=np.int32)
        cu = np.zeros(B + 1, dtype=np.int32)
        kv_lens = np.empty(B, dtype=np.int32)
        max_pages = max((e + 63) // 64 for _, _, e in chunks)
        bt = np.zeros((B, max_pages), dtype=np.int32)
        logits_rows, sample_reqs = [], []
        embeds, mm_rows, mm_list, ds_items = [], [], [], []
        any_embeds = any(r.input_embeds is not None for r, _, _ in chunks)
        off = 0
        for b, (r, s, e) in enumerate(chunks):
            n = e - s
            ids[off:off + n] = np.asarray(r.prefill_ids(s, e), dtype=np.int32)
            pos[:, off:off + n] = self._pos_rows(r, s, e)
            pages = np.asarray(r.pages, dtype=np.int64)
            t = np.arange(s, e)
            slots[off:off + n] = pages[t // 64] * 64 + (t % 64)
            cu[b + 1] = cu[b] + n
            kv_lens[b] = e
            bt[b, :len(r.pages)] = r.pages[:max_pages]
            if any_embeds:
                if r.input_embeds is not None:
                    embeds.append(h2d(adopt(r.input_embeds)[s:e], dev))
                else:
                    embeds.append(None)
            if r.mm_index is not None:
                mi = r.mm_index[s:e].clone()
                mm_rows.append((off, mi, r.mm_embeds))
            if r.deepstack is not None and r.ds_positions is not None:
                ds_items.append((off, s, e, r))
            if e >= r.prompt_len:
                logits_rows.append(off + n - 1)
                sample_reqs.append(r)
            off += n
        G = self.cfg.num_heads // self.cfg.num_kv_heads
        rows = prefill_tile_rows(self.cfg.head_dim, G) if self.is_cuda else 64
        req_t, tok0_t = prefill_tiles(q_lens, G, rows)
        as_dev = lambda a: h2d(a, dev)  # noqa: E731
        if any_embeds:
            parts = []
            for (r, s, e), emb in zip(chunks, embeds):
                if emb is None:
                    ids_d = h2d(ids[cu[len(parts)]:cu[len(parts)] + (e - s)], dev)
                    emb = self.model.embed[ids_d.long()]
                parts.append(emb.to(self.cfg.dtype))
            input_embeds = torch.cat(parts, 0)
        else:
            input_embeds = None
        mm_index = mm_embeds = None
        if mm_rows:
            mm_index_np = np.full(T, -1, dtype=np.int32)
            mats, base = [], 0
            for o, mi, emb in mm_rows:
                mi = mi.numpy().astype(np.int32)
                sel = mi >= 0
                mm_index_np[o:o + len(mi)][sel] = mi[sel] + base
                mats.append(emb)
                base += emb.shape[0]
            mm_index = as_dev(mm_index_np)
            mm_embeds = torch.cat([h2d(adopt(m), dev) for m in mats], 0).to(self.cfg.dtype)
        deepstack = None
        if ds_items:
            nl = max(len(r.deepstack) for *_, r in ds_items)
            deepstack = []
            for li in range(nl):
                ps, es = [], []
                for o, s, e, r in ds_items:
                    if li >= len(r.deepstack):
                        continue
                    p = r.ds_positions.long()
                    sel = (p >= s) & (p < e)
                    if bool(sel.any()):
                        ps.append(p[sel] - s + o)
                        es.append(r.deepstack[li][sel.nonzero().squeeze(1)])
                deepstack.append((h2d(torch.cat(ps), dev), h2d(torch.cat(es), dev)) if ps else None)
        capture = tuple(sorted({c for r, _, _ in chunks for c in r.capture_layers} |
                               {r.capture_prompt_layer for r, _, _ in chunks if r.capture_prompt_layer is not None}))
        fb = ForwardBatch(
            is_decode=False, positions=as_dev(pos), slot_mapping=as_dev(slots), kv_lens=as_dev(kv_lens),
            block_table=as_dev(bt), input_ids=as_dev(ids) if input_embeds is None else None,
            input_embeds=input_embeds, cu_q=as_dev(cu), tile_req=h2d(req_t, dev, torch.int32),
            tile_tok0=h2d(tok0_t, dev, torch.int32), tile_rows=rows,
            logits_indices=as_dev(np.asarray(logits_rows, dtype=np.int32)) if logits_rows else None,
            mm_index=mm_index, mm_embeds=mm_embeds, deepstack=deepstack, capture_layers=capture,
        )
        if not logits_rows:
            fb.logits_indices = torch.zeros(1, dtype=torch.int32, device=dev)
        hidden = self.model(fb, self.pool.kv)
        for b, (r, s, e) in enumerate(chunks):
            if r.capture_prompt_layer is not None and r.capture_prompt_layer in fb.captured:
                rows = fb.captured[r.capture_prompt_layer][cu[b]:cu[b + 1]]
                r.extra.setdefault("prompt_hidden", []).append(rows)
        captured = {}
        if capture and logits_rows:
            sel = fb.logits_indices.long()
            captured = {k: v[sel] for k, v in fb.captured.items()}
            captured["_full"] = fb.captured
            captured["_cu"] = cu
        if not logits_rows:
            return None
        row_slot = h2d([r.slot for r in sample_reqs], dev, torch.int32)
        toks = self._sample(hidden, row_slot)
        n = len(sample_reqs)
        host = self._next_tok_host()[:n]
        host.copy_(toks, non_blocking=True)
        ev = torch.cuda.Event() if self.is_cuda else None
        if ev is not None:
            ev.record()
        return {"reqs": sample_reqs, "host": host, "event": ev, "hidden": hidden, "captured": captured,
                "last_hidden": hidden}

    # ------------------------------------------------------------------ decode
    def _bucket(self, n: int) -> int:
        for b in self.buckets:
            if b >= n:
                return b
        raise ValueError(f"decode batch {n} exceeds max_batch {self.max_batch}")

    def _views(self, PB: int):
        P = self.max_pages
        m = self.meta_dev
        kv_lens = m[0:PB]
        slot_mapping = m[PB:2 * PB]
        positions = m[2 * PB:5 * PB].view(3, PB)
        slots = m[5 * PB:6 * PB]
        bt = m[6 * PB:6 * PB + PB * P].view(PB, P)
        return kv_lens, slot_mapping, positions, slots, bt

    def _decode_body(self, PB: int):
        kv_lens, slot_mapping, positions, slots, bt = self._views(PB)
        ids = self.slot_tokens[slots.long()]
        fb = ForwardBatch(is_decode=True, positions=positions, slot_mapping=slot_mapping, kv_lens=kv_lens,
                          block_table=bt, input_ids=ids, capture_layers=self._capture_layers)
        hidden = self.model(fb, self.pool.kv)
        toks = self._sample(hidden, slots)
        return toks, hidden, fb.captured

    def _sample(self, hidden: torch.Tensor, row_slot: torch.Tensor) -> torch.Tensor:
        """LM head + sampling (the model's vocab-parallel path under TP)."""
        fn = getattr(self.model, "sample_tokens", None)
        if fn is not None:
            return fn(hidden, self.st, self.suppress, row_slot=row_slot, slot_tokens=self.slot_tokens)
        return sample(self.model.logits(hidden), self.st, self.suppress, row_slot=row_slot,
                      slot_tokens=self.slot_tokens)

    _capture_layers: tuple = ()

    def set_capture_layers(self, layers: tuple):
        if tuple(layers) != self._capture_layers:
            self._capture_layers = tuple(layers)
            self.graphs.clear()

    def _fill_meta(self, reqs: list[ARRequest], PB: int):
        B = len(reqs)
        P = self.max_pages
        host = self.meta_ring.next().numpy()
        kl = np.fromiter((r.num_cached for r in reqs), dtype=np.int64, count=B)
        md = np.fromiter((r.mrope_delta for r in reqs), dtype=np.int64, count=B)
        sl = np.fromiter((r.slot for r in reqs), dtype=np.int64, count=B)
        if self.builder is not None:
            self.builder.build(host, [r.pages for r in reqs], kl, md, sl, self.pool.allocator_native(), PB)
        else:
            for i, r in enumerate(reqs):
                pos = int(kl[i])
                if pos // 64 >= len(r.pages):
                    r.pages.extend(self.pool.alloc(1))
            host[:6 * PB + PB * P] = 0
            host[0:B] = kl + 1
            host[PB:PB + B] = [r.pages[int(k) // 64] * 64 + int(k) % 64 for r, k in zip(reqs, kl)]
            host[PB + B:2 * PB] = -1
            for j in range(3):
                host[(2 + j) * PB:(2 + j) * PB + B] = kl + md
            host[5 * PB:5 * PB + B] = sl
            for i, r in enumerate(reqs):
                host[6 * PB + i * P:6 * PB + i * P + len(r.pages)] = r.pages
        n = 6 * PB + PB * P
        self.meta_ring.upload(self.meta_dev, n)

    def capture_all(self):
        """Captures the decode graph of every batch bucket up front."""
        if self.use_graphs:
            for PB in self.buckets:
                self.capture(PB)

    @torch.no_grad()
    def capture(self, PB: int):
        if not self.use_graphs or PB in self.graphs:
            return
        # dummy-but-valid metadata: every row is padding (empty context, no cache write)
        host = self.meta_ring.next().numpy()
        n = 6 * PB + PB * self.max_pages
        host[:n] = 0
        host[PB:2 * PB] = -1
        self.meta_ring.upload(self.meta_dev, n, blocking=True)
        self.graphs[PB] = capture_graph(lambda: self._decode_body(PB))

    @torch.no_grad()
    def decode(self, reqs: list[ARRequest]):
        B = len(reqs)
        PB = self._bucket(B)
        self._fill_meta(reqs, PB)
        for r in reqs:
            r.num_cached += 1
            r.scheduled_decodes += 1
        if self.use_graphs:
            if PB not in self.graphs:
                self.capture(PB)
                self._fill_meta_restore(reqs, PB)
            g, (toks, hidden, captured) = self.graphs[PB]
            g.replay()
        else:
            toks, hidden, captured = self._decode_body(PB)
        host = self._next_tok_host()[:B]
        host.copy_(toks[:B], non_blocking=True)
        ev = torch.cuda.Event() if self.is_cuda else None
        if ev is not None:
            ev.record()
        cap = {k: v[:B] for k, v in captured.items()} if self._capture_layers else {}
        return {"reqs": list(reqs), "host": host, "event": ev, "hidden": hidden[:B], "captured": cap}

    def _fill_meta_restore(self, reqs, PB):
        # capture() overwrote the metadata with padding; rebuild it without re-allocating pages
        B = len(reqs)
        saved = [(r.num_cached, r.scheduled_decodes) for r in reqs]
        for r in reqs:
            r.num_cached -= 1
        self._fill_meta(reqs, PB)
        for r, (nc, sd) in zip(reqs, saved):
            r.num_cached, r.scheduled_decodes = nc, sd
