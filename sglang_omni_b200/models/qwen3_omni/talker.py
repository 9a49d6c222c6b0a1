"""Qwen3-Omni talker + code predictor, batched across speech streams.

Talker: MoE decoder (20 layers, 128 experts top-6 + sigmoid-gated shared
expert) over projected thinker states; its codec head samples the layer-0
code of each 12.5 Hz frame.  Code predictor: 5-layer dense decoder that, per
frame, extends [talker_hidden, embed0(code0)] autoregressively with 15
codebook-specific heads / embeddings; the sum of the 16 code embeddings is fed
back as the next talker input (plus the next projected thinker text state, or
``tts_pad``).

``SpeechGenerator`` runs all active streams in lock step: one talker decode
step + the 16 code-predictor sub-steps (talker hidden, then one per code
group) are captured together in ONE CUDA graph per batch bucket, so the
talker <-> code-predictor feedback loop never leaves the GPU and costs one
graph launch per frame.  Per-stream state (feedback embedding, projected
trailing text, step counters, sampling state) lives in fixed per-slot device
buffers.

Reference counterparts: Qwen3OmniTalker / code_predictor_forward
(sglang_omni/models/qwen3_omni/talker.py:65-953), the HF-parity prefill
builder (sglang_omni/models/qwen3_omni/components/talker_input.py:8-269), the
talker streaming executor and code-predictor stage
(sglang_omni/models/qwen3_omni/components/talker_executor.py,
code_predictor_executor.py).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch
from torch import nn

from ... import ops
from ...engines.ar.kv_pool import KVPool
from ...ops.sampling import SamplingTensors, sample
from ...environ import environ
from ...utils.cuda_graph import capture_graph
from ...utils.hostdev import h2d
from ...utils.staging import PinnedRing
from ..decoder import DecoderConfig, DecoderLM, ForwardBatch
from .hf_config import code_predictor_config, talker_text_config


@dataclass
class TalkerSpecialTokens:
    codec_eos: int = 2150
    codec_nothink: int = 2155
    codec_think_bos: int = 2156
    codec_think_eos: int = 2157
    codec_pad: int = 2148
    codec_bos: int = 2149
    speakers: dict = field(default_factory=lambda: {"chelsie": 2301, "ethan": 2302, "aiden": 2303})
    default_speaker: str = "ethan"
    tts_pad: int = 151671
    tts_bos: int = 151672
    tts_eos: int = 151673
    im_start: int = 151644
    im_end: int = 151645
    system: int = 8948
    user: int = 872
    assistant: int = 77091
    newline: int = 198
    accept_hidden_layer: int = 24
    num_code_groups: int = 16


class Qwen3OmniTalker(nn.Module):
    def __init__(self, tcfg: DecoderConfig | None = None, cpcfg: DecoderConfig | None = None,
                 thinker_hidden: int = 2048, special: TalkerSpecialTokens | None = None, device="cpu"):
        super().__init__()
        tcfg = tcfg or talker_text_config()
        cpcfg = cpcfg or code_predictor_config()
        cpcfg.tie_word_embeddings = True
        self.special = special or TalkerSpecialTokens()
        self.lm = DecoderLM(tcfg, device)          # embed = codec_embedding, lm_head = codec_head
        self.cp = DecoderLM(cpcfg, device)
        H, dt, I = tcfg.hidden_size, tcfg.dtype, tcfg.intermediate_size
        P = lambda *s: nn.Parameter(torch.empty(*s, dtype=dt, device=device), requires_grad=False)  # noqa: E731
        self.text_fc1_w, self.text_fc1_b = P(I, thinker_hidden), P(I)
        self.text_fc2_w, self.text_fc2_b = P(H, I), P(H)
        self.hid_fc1_w, self.hid_fc1_b = P(I, thinker_hidden), P(I)
        self.hid_fc2_w, self.hid_fc2_b = P(H, I), P(H)
        G = self.special.num_code_groups - 1
        self.cp_embeds = P(G, cpcfg.vocab_size, cpcfg.hidden_size)
        self.cp_heads = P(G, cpcfg.vocab_size, cpcfg.hidden_size)

    @torch.no_grad()
    def random_init_(self, seed: int = 0, std: float = 0.02):
        self.lm.random_init_(seed * 3 + 1, std)
        self.cp.random_init_(seed * 3 + 2, std)
        dev = self.text_fc1_w.device
        for idx, (n, p) in enumerate(self.named_parameters(recurse=False)):
            if n.endswith("_b"):
                p.zero_()
            else:
                g = torch.Generator(device=dev).manual_seed(seed * 1009 + idx)
                p.normal_(0.0, std, generator=g)
        return self

    def project_text(self, x: torch.Tensor) -> torch.Tensor:
        return ops.linear(ops.linear(x, self.text_fc1_w, bias=self.text_fc1_b, act="silu"), self.text_fc2_w,
                          bias=self.text_fc2_b)

    def project_hidden(self, x: torch.Tensor) -> torch.Tensor:
        return ops.linear(ops.linear(x, self.hid_fc1_w, bias=self.hid_fc1_b, act="silu"), self.hid_fc2_w,
                          bias=self.hid_fc2_b)

    def codec_embed(self, ids: torch.Tensor) -> torch.Tensor:
        return self.lm.embed[ids.long()]


# ----------------------------------------------------------------------------- prefill input (HF parity)
def segment_chat_template(ids: list[int], sp: TalkerSpecialTokens) -> list[tuple[str, int, int]]:
    roles = {sp.system: "system", sp.user: "user", sp.assistant: "assistant"}
    starts = [i for i, t in enumerate(ids) if t == sp.im_start]
    segs = []
    for n, s in enumerate(starts):
        role = roles.get(ids[s + 1] if s + 1 < len(ids) else -1, "unknown")
        e = starts[n + 1] if n + 1 < len(starts) else len(ids)
        segs.append((role, s, e))
    return segs


def build_talker_prefill(talker: Qwen3OmniTalker, thinker_embed: torch.Tensor, prompt_ids: list[int],
                         first_tokens: list[int], mm_mask: torch.Tensor | None = None,
                         mm_hidden: torch.Tensor | None = None, speaker: str | None = None):
    """Returns (prefill input_embeds [L, H], trailing projected text [n, H]).

    User segments: text positions -> text projection of the thinker token
    embedding, multimodal positions -> hidden projection of the thinker's
    accept-layer state.  Assistant segment (the last one, i.e. the response):
    [3 template tokens, 4 x tts_pad, tts_bos, 1st response token] on the text
    side plus [0, 0, 0, nothink, think_bos, think_eos, speaker, pad, bos] codec
    embeddings; the remaining response tokens become the trailing text.
    """
    sp = talker.special
    dev = thinker_embed.device
    ids = list(prompt_ids)
    segs = segment_chat_template(ids, sp)
    parts = []
    pad_e, bos_e, eos_e = talker.project_text(thinker_embed[h2d([sp.tts_pad, sp.tts_bos, sp.tts_eos], dev,
                                                                 torch.long)]).split(1, 0)
    mm_cpu = None if mm_mask is None else mm_mask.cpu() if mm_mask.is_cuda else mm_mask
    for role, s, e in segs:
        if role != "user":
            continue
        emb = talker.project_text(thinker_embed[h2d(ids[s:e], dev, torch.long)])
        if mm_cpu is not None and mm_hidden is not None:
            sel = mm_cpu[s:e].nonzero().view(-1)           # host-side: no device sync
            if sel.numel():
                rows = mm_hidden[s:e].index_select(0, h2d(sel, mm_hidden.device))
                emb.index_copy_(0, h2d(sel, dev), talker.project_hidden(rows.to(dev)).to(emb.dtype))
        parts.append(emb)
    # assistant part: the template tokens "<|im_start|>assistant\n" then the response
    asst = [sp.im_start, sp.assistant, sp.newline] + list(first_tokens)
    proj = talker.project_text(thinker_embed[h2d(asst, dev, torch.long)])
    fourth = proj[3:4] if proj.shape[0] > 3 else torch.zeros_like(proj[:1])
    text_side = torch.cat([proj[:3], pad_e.expand(4, -1), bos_e, fourth], 0)
    spk = sp.speakers.get((speaker or sp.default_speaker).lower(), next(iter(sp.speakers.values())))
    codec_ids = h2d([sp.codec_nothink, sp.codec_think_bos, sp.codec_think_eos, spk, sp.codec_pad, sp.codec_bos],
                    dev, torch.long)
    codec_side = torch.cat([torch.zeros(3, proj.shape[1], dtype=proj.dtype, device=dev),
                            talker.codec_embed(codec_ids).to(proj.dtype)], 0)
    parts.append(text_side + codec_side)
    trailing = proj[4:]
    return torch.cat(parts, 0), trailing, pad_e[0], eos_e[0]


# ----------------------------------------------------------------------------- batched runtime
@dataclass
class SpeechStream:
    rid: str
    slot: int
    pages: list = field(default_factory=list)
    num_cached: int = 0
    steps: int = 0                 # talker decode steps done (frames after the first)
    trailing_len: int = 0          # projected trailing text states available in the device buffer
    thinker_done: bool = False
    finished: bool = False
    frames: int = 0
    max_frames: int = 4096
    eos_written: bool = False


class SpeechGenerator:
    """Talker + code predictor for many concurrent streams (single GPU)."""

    def __init__(self, talker: Qwen3OmniTalker, thinker_embed: torch.Tensor, max_streams: int = 64,
                 max_context: int = 2048, max_trailing: int = 1024, use_graphs: bool = True,
                 talker_sampling=(0.9, 50, 1.0, 1.05), cp_sampling=(1.0, 50, 0.8), seed: int = 0,
                 tail_frames: int = 50):
        self.talker = talker
        self.thinker_embed = thinker_embed
        tc, cc = talker.lm.cfg, talker.cp.cfg
        dev = thinker_embed.device
        self.device = dev
        self.sp = talker.special
        self.G = self.sp.num_code_groups
        self.max_streams = max_streams
        self.max_pages = (max_context + 63) // 64
        self.pool = KVPool(tc.num_layers, tc.num_kv_heads, tc.head_dim, max_streams * self.max_pages + 2, dev,
                           tc.dtype)
        # one CP page per slot (16 tokens <= 64)
        self.cp_pool = KVPool(cc.num_layers, cc.num_kv_heads, cc.head_dim, max_streams + 2, dev, cc.dtype)
        talker.lm.ensure_workspaces(max(max_streams, 512) * 8, max_streams, max_context)
        talker.cp.ensure_workspaces(max_streams, max_streams, 64)
        S = max_streams + 1  # slot 0 = padding
        H = tc.hidden_size
        self.feedback = torch.zeros(S, H, dtype=tc.dtype, device=dev)
        self.trail = torch.zeros(S, max_trailing + 2, H, dtype=tc.dtype, device=dev)
        self.trail_idx = torch.zeros(S, dtype=torch.long, device=dev)
        self.pad_embed = torch.zeros(H, dtype=tc.dtype, device=dev)
        self.max_trailing = max_trailing
        # after the thinker finished and its text is consumed, a stream that
        # has not produced the codec EOS stops after tail_frames more frames
        self.tail_frames = tail_frames
        # sampling state (talker: rows = slots; CP: rows = slots, 15 groups share it)
        t, k, p, rep = talker_sampling
        self.t_st = SamplingTensors(torch.full((S,), t, device=dev), torch.full((S,), k, dtype=torch.int32, device=dev),
                                    torch.full((S,), p, device=dev), torch.zeros(S, device=dev),
                                    torch.full((S,), rep, device=dev),
                                    torch.zeros(S, tc.vocab_size, dtype=torch.uint8, device=dev),
                                    torch.arange(S, dtype=torch.int64, device=dev) * 7919 + seed,
                                    torch.zeros(S, dtype=torch.int32, device=dev))
        ct, ck, cpp = cp_sampling
        self.c_st = SamplingTensors(torch.full((S,), ct, device=dev),
                                    torch.full((S,), ck, dtype=torch.int32, device=dev),
                                    torch.full((S,), cpp, device=dev), None, None, None,
                                    torch.arange(S, dtype=torch.int64, device=dev) * 104729 + seed,
                                    torch.zeros(S, dtype=torch.int32, device=dev))
        self.code0_tok = torch.zeros(S, dtype=torch.int32, device=dev)
        self.cp_tok = torch.zeros(S, dtype=torch.int32, device=dev)
        self.suppress = (tc.vocab_size - 1024, tc.vocab_size, self.sp.codec_eos)
        self.streams: dict[str, SpeechStream] = {}
        self.free_slots = list(range(S - 1, 0, -1))
        self.use_graphs = use_graphs and dev.type == "cuda" and environ.OMNI_USE_CUDA_GRAPHS.get()
        self.graphs: dict[int, tuple] = {}
        self.buckets = [b for b in (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128) if b <= max_streams]
        if self.buckets[-1] < max_streams:
            self.buckets.append(max_streams)
        PB = max_streams
        self.meta_ring = PinnedRing(6 * PB + PB * self.max_pages, torch.int32, 2, dev.type == "cuda")
        self.meta_dev = torch.zeros(6 * PB + PB * self.max_pages, dtype=torch.int32, device=dev)
        self.codes_out = torch.zeros(S, self.G, dtype=torch.int32, device=dev)
        try:
            from ... import _runtime as rt
            self.builder = rt.DecodeMetaBuilder(PB, self.max_pages)
        except ImportError:  # pragma: no cover
            self.builder = None

    # ------------------------------------------------------------------ stream management
    def add_stream(self, rid: str, prefill_embeds: torch.Tensor, trailing: torch.Tensor, pad_e, eos_e,
                   thinker_done: bool = False, max_frames: int = 4096) -> SpeechStream:
        slot = self.free_slots.pop()
        # the KV of prefill + one position per frame must fit the slot's pages
        max_frames = max(1, min(max_frames, self.max_pages * 64 - prefill_embeds.shape[0]))
        st = SpeechStream(rid, slot, max_frames=max_frames)
        self.streams[rid] = st
        self.pad_embed.copy_(pad_e)
        self._eos_embed = eos_e
        self.trail[slot].copy_(pad_e.expand_as(self.trail[slot]))
        self.trail_idx[slot] = 0
        self.t_st.seen[slot].zero_()
        self.t_st.step[slot] = 0
        self.c_st.step[slot] = 0
        self.push_trailing(rid, trailing, thinker_done)
        st._prefill = prefill_embeds
        return st

    def push_trailing(self, rid: str, projected: torch.Tensor | None, done: bool = False) -> None:
        st = self.streams[rid]
        if projected is not None and projected.shape[0]:
            n = min(projected.shape[0], self.max_trailing - st.trailing_len)
            self.trail[st.slot, st.trailing_len:st.trailing_len + n] = projected[:n]
            st.trailing_len += n
        if done and not st.thinker_done:
            st.thinker_done = True
            if st.trailing_len < self.max_trailing:
                self.trail[st.slot, st.trailing_len] = self._eos_embed
                st.trailing_len += 1
            st.max_frames = min(st.max_frames, st.trailing_len + self.tail_frames)

    def remove(self, rid: str) -> None:
        st = self.streams.pop(rid, None)
        if st is not None:
            self.pool.free(st.pages)
            self.free_slots.append(st.slot)

    def ready_streams(self) -> list[SpeechStream]:
        return [s for s in self.streams.values() if not s.finished and not hasattr(s, "_prefill")
                and (s.steps < s.trailing_len or s.thinker_done)]

    # ------------------------------------------------------------------ code predictor
    def _code_predictor(self, hidden: torch.Tensor, slots: torch.Tensor, code0: torch.Tensor, cp_bt, cp_slot_base):
        """15 codebook steps for B rows. Returns (codes [B, G] int32, summed embeds [B, H])."""
        tl, cp = self.talker.lm, self.talker.cp
        B = hidden.shape[0]
        dev = hidden.device
        e0 = tl.embed[code0.long()]
        summed = e0.float()
        codes = [code0]
        x = hidden
        for j in range(self.G):  # token j of the CP sequence: 0 = talker hidden, 1 = embed0, ...
            pos = torch.full((B,), j, dtype=torch.int32, device=dev)
            kv_lens = torch.full((B,), j + 1, dtype=torch.int32, device=dev)
            fb = ForwardBatch(is_decode=True, positions=pos, slot_mapping=cp_slot_base + j, kv_lens=kv_lens,
                              block_table=cp_bt, input_embeds=x)
            h = cp(fb, self.cp_pool.kv)
            if j == 0:
                x = e0
                continue
            g = j - 1
            logits = ops.linear(h, self.talker.cp_heads[g], out_dtype=torch.float32)
            c = sample(logits, self.c_st, row_slot=slots, slot_tokens=self.cp_tok)
            codes.append(c)
            emb = self.talker.cp_embeds[g][c.long()]
            summed = summed + emb.float()
            x = emb
        return torch.stack(codes, 1), summed.to(hidden.dtype)

    def _talker_tail(self, hidden: torch.Tensor, slots: torch.Tensor, cp_bt, cp_slot_base):
        logits = ops.linear(hidden, self.talker.lm.head_weight, out_dtype=torch.float32)
        code0 = sample(logits, self.t_st, self.suppress, row_slot=slots, slot_tokens=self.code0_tok)
        codes, summed = self._code_predictor(hidden, slots, code0, cp_bt, cp_slot_base)
        self.feedback[slots.long()] = summed
        self.codes_out[slots.long()] = codes
        return codes

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, streams: list[SpeechStream]):
        if not streams:
            return None
        dev = self.device
        tl = self.talker.lm
        embeds = [s._prefill for s in streams]
        lens = [e.shape[0] for e in embeds]
        for s, n in zip(streams, lens):
            need = KVPool.pages_for(n) - len(s.pages)
            if need > 0:
                s.pages.extend(self.pool.alloc(need))
        T = sum(lens)
        cu = np.zeros(len(streams) + 1, dtype=np.int32)
        cu[1:] = np.cumsum(lens)
        pos = np.concatenate([np.arange(n, dtype=np.int32) for n in lens])
        slot_map = np.concatenate([np.asarray(s.pages)[np.arange(n) // 64] * 64 + np.arange(n) % 64
                                   for s, n in zip(streams, lens)]).astype(np.int32)
        bt = np.zeros((len(streams), max(len(s.pages) for s in streams)), dtype=np.int32)
        for i, s in enumerate(streams):
            bt[i, :len(s.pages)] = s.pages
        G = tl.cfg.num_heads // tl.cfg.num_kv_heads
        rows = ops.prefill_tile_rows(tl.cfg.head_dim, G) if dev.type == "cuda" else 64
        req, tok0 = ops.prefill_tiles(lens, G, rows)
        d = lambda a: h2d(a, dev)  # noqa: E731
        fb = ForwardBatch(is_decode=False, positions=d(np.stack([pos] * 3)), slot_mapping=d(slot_map),
                          kv_lens=h2d(lens, dev, torch.int32), block_table=d(bt),
                          input_embeds=torch.cat(embeds, 0).to(tl.cfg.dtype), cu_q=d(cu),
                          tile_req=h2d(req, dev, torch.int32), tile_tok0=h2d(tok0, dev, torch.int32),
                          tile_rows=rows, logits_indices=d(cu[1:] - 1))
        hidden = tl(fb, self.pool.kv)
        slots = h2d([s.slot for s in streams], dev, torch.int32)
        cp_bt = (slots + 1).view(-1, 1).to(torch.int32)
        cp_base = (slots + 1) * 64
        codes = self._talker_tail(hidden, slots, cp_bt, cp_base)
        for s, n in zip(streams, lens):
            s.num_cached = n
            s.frames = 1
            del s._prefill
        return codes

    # ------------------------------------------------------------------ decode step
    def _bucket(self, n):
        for b in self.buckets:
            if b >= n:
                return b
        raise ValueError(n)

    def _views(self, PB):
        m = self.meta_dev
        P = self.max_pages
        return (m[0:PB], m[PB:2 * PB], m[2 * PB:5 * PB].view(3, PB), m[5 * PB:6 * PB],
                m[6 * PB:6 * PB + PB * P].view(PB, P))

    def _step_body(self, PB):
        kv_lens, slot_mapping, positions, slots, bt = self._views(PB)
        sl = slots.long()
        inp = self.feedback[sl] + self.trail[sl, self.trail_idx[sl]]
        fb = ForwardBatch(is_decode=True, positions=positions, slot_mapping=slot_mapping, kv_lens=kv_lens,
                          block_table=bt, input_embeds=inp)
        hidden = self.talker.lm(fb, self.pool.kv)
        cp_bt = (slots + 1).view(-1, 1)
        cp_base = (slots + 1) * 64
        self.trail_idx[sl] = torch.clamp(self.trail_idx[sl] + 1, max=self.max_trailing)
        return self._talker_tail(hidden, slots, cp_bt, cp_base)

    def _fill_meta(self, streams, PB):
        host = self.meta_ring.next().numpy()
        B = len(streams)
        kl = np.fromiter((s.num_cached for s in streams), dtype=np.int64, count=B)
        md = np.zeros(B, dtype=np.int64)
        sl = np.fromiter((s.slot for s in streams), dtype=np.int64, count=B)
        self.builder.build(host, [s.pages for s in streams], kl, md, sl, self.pool.allocator_native(), PB)
        n = 6 * PB + PB * self.max_pages
        self.meta_ring.upload(self.meta_dev, n)

    @torch.no_grad()
    def step(self, streams: list[SpeechStream]):
        """One frame for every stream in `streams`; returns codes [B, G] (device)."""
        B = len(streams)
        PB = self._bucket(B)
        if self.use_graphs and PB not in self.graphs:
            self._capture(PB)
        self._fill_meta(streams, PB)
        if self.use_graphs:
            g, codes = self.graphs[PB]
            g.replay()
        else:
            codes = self._step_body(PB)
        for s in streams:
            s.num_cached += 1
            s.steps += 1
            s.frames += 1
        return codes[:B]

    def capture_all(self):
        """Captures the frame-step graph of every batch bucket up front."""
        if self.use_graphs:
            for PB in self.buckets:
                if PB not in self.graphs:
                    self._capture(PB)

    def _capture(self, PB):
        host = self.meta_ring.next().numpy()
        n = 6 * PB + PB * self.max_pages
        host[:n] = 0
        host[PB:2 * PB] = -1
        self.meta_ring.upload(self.meta_dev, n, blocking=True)
        saved = (self.feedback.clone(), self.trail_idx.clone(), self.codes_out.clone(), self.t_st.step.clone(),
                 self.c_st.step.clone(), self.t_st.seen[0].clone())
        g, codes = capture_graph(lambda: self._step_body(PB))
        # padding rows only touched slot 0; restore the state rows they may have changed
        self.feedback.copy_(saved[0])
        self.trail_idx.copy_(saved[1])
        self.codes_out.copy_(saved[2])
        self.t_st.step.copy_(saved[3])
        self.c_st.step.copy_(saved[4])
        self.t_st.seen[0].copy_(saved[5])
        self.graphs[PB] = (g, codes)
