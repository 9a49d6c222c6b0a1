"""Decoder-only transformer shared by every autoregressive stage.

One implementation covers:
  * the Qwen3-Omni thinker (MoE 128x top-8, QK-norm, interleaved M-RoPE),
  * the Qwen3-Omni talker (MoE top-6 + sigmoid-gated shared expert),
  * the Qwen3-Omni code predictor (dense SwiGLU),
  * the S2-Pro slow AR (dense, non-neox RoPE, tied embeddings),
  * Ming's BailingMoeV2 LLM (sigmoid group-limited routing, partial RoPE,
    first-k dense layers, shared expert).

All hot ops go through ``sglang_omni_b200.ops`` (sm_100a kernels on CUDA,
PyTorch restatements on CPU).  Fused weight layouts: ``qkv`` = [q; k; v],
``w13`` = [gate; up] per expert, so the SiLU*up multiply happens inside the
GEMM epilogue.

Reference counterparts: Qwen3OmniMoeThinkerTextModel / DecoderLayer /
Attention / SparseMoeBlock (sglang_omni/models/qwen3_omni/thinker.py:140-706),
the talker text model (sglang_omni/models/qwen3_omni/talker.py:177-400), the
S2-Pro SGLang text model (sglang_omni/models/fishaudio_s2_pro/sglang_model.py:53-380)
and BailingMoeV2 (sglang_omni/models/ming_omni/thinker.py:155-826).
"""
from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass, field

import torch
from torch import nn

from .. import ops
from ..ops.attention import DecodeWorkspace
from ..ops.gemm import static_weights
from ..ops.moe import MoEWorkspace


@dataclass
class DecoderConfig:
    vocab_size: int = 151936
    hidden_size: int = 2048
    num_layers: int = 48
    num_heads: int = 32
    num_kv_heads: int = 4
    head_dim: int = 128
    intermediate_size: int = 0          # dense SwiGLU width (dense layers)
    num_experts: int = 0
    topk: int = 0
    moe_intermediate_size: int = 0
    shared_expert_intermediate_size: int = 0
    shared_expert_gate: bool = True     # sigmoid gate on the shared expert (Qwen3 talker)
    norm_topk_prob: bool = True
    router_mode: int = 0                # 0 softmax top-k, 1 sigmoid + bias group-limited
    n_group: int = 1
    topk_group: int = 1
    routed_scaling_factor: float = 1.0
    first_k_dense: int = 0
    mlp_only_layers: tuple = ()
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    rope_scaling: dict | None = None    # HF rope_scaling: linear / llama3 frequency rescaling
    rope_neox: bool = True
    rotary_dim: int | None = None
    mrope_section: list | None = None   # e.g. [24, 20, 20]
    mrope_interleaved: bool = True
    qk_norm: bool = True
    attention_bias: bool = False        # q / k / v projection biases (Qwen2)
    tie_word_embeddings: bool = False
    max_position: int = 65536
    dtype: torch.dtype = torch.bfloat16
    name: str = "decoder"

    def is_moe_layer(self, i: int) -> bool:
        return self.num_experts > 0 and i >= self.first_k_dense and i not in self.mlp_only_layers

    @property
    def q_size(self):
        return self.num_heads * self.head_dim

    @property
    def kv_size(self):
        return self.num_kv_heads * self.head_dim

    def param_count(self) -> int:
        H = self.hidden_size
        n = 2 * self.vocab_size * H if not self.tie_word_embeddings else self.vocab_size * H
        for i in range(self.num_layers):
            n += H * (self.q_size + 2 * self.kv_size) + self.q_size * H + 2 * H
            if self.is_moe_layer(i):
                n += self.num_experts * (3 * H * self.moe_intermediate_size) + self.num_experts * H
                if self.shared_expert_intermediate_size:
                    n += 3 * H * self.shared_expert_intermediate_size + H
            else:
                n += 3 * H * self.intermediate_size
        return n


@dataclass
class ForwardBatch:
    """Device-side description of one engine step (prefill chunk or decode)."""

    is_decode: bool
    positions: torch.Tensor                 # int32 [3, T] (M-RoPE) or [T]
    slot_mapping: torch.Tensor | None       # int32 [T]
    kv_lens: torch.Tensor                   # int32 [B]
    block_table: torch.Tensor               # int32 [B, max_pages]
    input_ids: torch.Tensor | None = None   # int32 [T]
    input_embeds: torch.Tensor | None = None
    cu_q: torch.Tensor | None = None        # prefill: int32 [B + 1]
    tile_req: torch.Tensor | None = None
    tile_tok0: torch.Tensor | None = None
    tile_rows: int = 64                     # packed rows per prefill tile (ops.prefill_tile_rows)
    logits_indices: torch.Tensor | None = None  # rows whose logits are needed
    mm_index: torch.Tensor | None = None    # int32 [T] row of mm_embeds or -1
    mm_embeds: torch.Tensor | None = None
    deepstack: list | None = None           # [(positions int64 [n], embeds [n, H])] for layers 0..
    capture_layers: tuple = ()
    captured: dict = field(default_factory=dict)


class DecoderLM(nn.Module):
    """Weights as plain parameters in fused layouts; forward is op-by-op on the kernels."""

    def __init__(self, cfg: DecoderConfig, device="cpu", ep=None, tp=None, vocab_parallel: bool = True,
                 vocab_cand: int = 64):
        """``ep``: an ``parallel.EPMoE`` exchange; this rank then holds experts
        [ep.rank * El, (ep.rank + 1) * El) and the MoE layers run expert-parallel.

        ``tp``: a ``parallel.TPGroup``; this rank then holds its query / KV heads
        (``self.cfg`` describes the local attention: local head counts), the
        matching o_proj columns, experts [rank * E / world, ...) and slices of the
        shared-expert / dense MLP intermediate; every rank runs every token and the
        reduce points are the fused peer-memory kernels of ``parallel.tp``.

        Both: attention and dense MLPs are tensor-parallel over ``tp`` and the MoE layers
        expert-parallel over ``ep`` (experts [ep.rank * El, ...), shared experts whole).
        After the o_proj reduce point each TP rank keeps the normalised rows it owns and
        dispatches only those, so every token crosses the EP exchange once; the EP
        combine writes the owned rows' expert output into the TP partial slot and the
        next reduce point adds the residual, normalises and all-gathers them.  With
        ep.world > tp.world the TP groups are data-parallel replicas of the attention."""
        super().__init__()
        self.full_cfg = cfg
        self.tp = tp
        self._tp_split = None
        if tp is not None:
            from ..parallel.tp import head_split

            qh, kvh = head_split(cfg.num_heads, cfg.num_kv_heads, tp.rank, tp.world)
            self._tp_split = (qh, kvh)
            assert ep is not None or cfg.num_experts % tp.world == 0 or not cfg.num_experts
            shared_w = cfg.shared_expert_intermediate_size
            for w in (cfg.intermediate_size, 0 if ep is not None else shared_w):
                assert w % tp.world == 0, "MLP widths must divide over the TP group"
            cfg = dataclasses.replace(cfg, num_heads=len(qh), num_kv_heads=len(kvh),
                                      intermediate_size=cfg.intermediate_size // tp.world,
                                      shared_expert_intermediate_size=shared_w if ep is not None
                                      else shared_w // tp.world)
        self.cfg = cfg
        self.ep = ep
        par = ep if ep is not None else tp
        self.num_local_experts = cfg.num_experts if par is None else cfg.num_experts // par.world
        self.expert0 = 0 if par is None else par.rank * self.num_local_experts
        H, dt = cfg.hidden_size, cfg.dtype
        P = lambda *shape: nn.Parameter(torch.empty(*shape, dtype=dt, device=device), requires_grad=False)  # noqa: E731
        self.embed = P(cfg.vocab_size, H)
        self.layers = nn.ModuleList()
        for i in range(cfg.num_layers):
            L = nn.Module()
            L.ln1 = P(H)
            L.qkv = P(cfg.q_size + 2 * cfg.kv_size, H)
            if cfg.attention_bias:   # under TP: the local heads' rows, as the QKV weight
                L.qkv_bias = P(cfg.q_size + 2 * cfg.kv_size)
            L.o = P(H, cfg.q_size)
            L.ln2 = P(H)
            if cfg.qk_norm:
                L.q_norm = P(cfg.head_dim)
                L.k_norm = P(cfg.head_dim)
            if cfg.is_moe_layer(i):
                E, I = cfg.num_experts, cfg.moe_intermediate_size
                L.router = P(E, H)
                L.w13 = P(self.num_local_experts, 2 * I, H)
                L.w2 = P(self.num_local_experts, H, I)
                if cfg.router_mode == 1:
                    L.router_bias = nn.Parameter(torch.zeros(E, dtype=torch.float32, device=device),
                                                 requires_grad=False)
                if cfg.shared_expert_intermediate_size:
                    Is = cfg.shared_expert_intermediate_size
                    L.s13 = P(2 * Is, H)
                    L.s2 = P(H, Is)
                    if cfg.shared_expert_gate:
                        L.sgate = P(1, H)
            else:
                L.mlp13 = P(2 * cfg.intermediate_size, H)
                L.mlp2 = P(H, cfg.intermediate_size)
            self.layers.append(L)
        self.final_norm = P(H)
        # Under TP the LM head is split over the vocabulary (rows [vocab0, vocab0 + vocab_local)
        # on this rank, zero-padded to a 16-multiple width) and tokens are drawn by the
        # vocab-parallel sampler (parallel/vocab.py) without gathering the logits.
        self.vocab_sampler = None
        self._vslice = (0, cfg.vocab_size, cfg.vocab_size)
        if tp is not None and vocab_parallel:
            from ..parallel.vocab import vocab_slice

            self._vslice = vocab_slice(cfg.vocab_size, tp.rank, tp.world)
        head_rows = self._vslice[2] if tp is not None and vocab_parallel else cfg.vocab_size
        self.lm_head = None if cfg.tie_word_embeddings else P(head_rows, H)
        rot = cfg.rotary_dim or cfg.head_dim
        cos, sin = ops.rope_tables(rot, cfg.rope_theta, cfg.max_position, device, round_bf16=cfg.dtype == torch.bfloat16,
                                   scaling=cfg.rope_scaling)
        self.register_buffer("cos_tab", cos, persistent=False)
        self.register_buffer("sin_tab", sin, persistent=False)
        self._moe_ws: MoEWorkspace | None = None
        self._dec_ws: DecodeWorkspace | None = None
        self._retired_ws: list = []
        if tp is not None and vocab_parallel and torch.device(device).type == "cuda":
            from ..parallel.vocab import VocabParallelSampler

            self.vocab_sampler = VocabParallelSampler(cfg.vocab_size, min(tp.max_tokens, 512), device,
                                                      group=tp.group, cand=vocab_cand, timeout_s=tp.timeout_s)

    # ------------------------------------------------------------------ init
    @torch.no_grad()
    def random_init_(self, seed: int = 0, std: float = 0.02):
        """N(0, std) for matrices, ones for norm weights; deterministic per parameter
        (per expert for expert weights, so an expert-parallel rank draws exactly its
        slice of the full model)."""
        dev = self.embed.device
        for idx, (name, p) in enumerate(self.named_parameters()):
            if p.dim() == 1 and ("ln" in name or "norm" in name):
                p.fill_(1.0)
            elif name.endswith(("router_bias", "qkv_bias")):
                p.zero_()
            elif name.endswith((".w13", ".w2")):
                for j in range(p.shape[0]):
                    g = torch.Generator(device=dev).manual_seed((seed * 100003 + idx) * 1009 + self.expert0 + j)
                    p[j].normal_(0.0, std, generator=g)
            else:
                g = torch.Generator(device=dev).manual_seed(seed * 100003 + idx)
                kind = name.rsplit(".", 1)[-1]
                full = self.full_shape(kind, p)
                if full is None:
                    p.normal_(0.0, std, generator=g)
                else:   # tensor parallel: draw the unsharded tensor, keep this rank's slice
                    t = torch.empty(full, dtype=p.dtype, device=dev).normal_(0.0, std, generator=g)
                    p.copy_(self.shard(kind, t))
        return self

    # ------------------------------------------------------------------ tensor-parallel slices
    _TP_KINDS = ("qkv", "qkv_bias", "o", "s13", "s2", "mlp13", "mlp2", "lm_head")

    def full_shape(self, kind: str, p: torch.Tensor):
        """Unsharded shape of a tensor-parallel parameter (None if not sharded)."""
        if self.tp is None or kind not in self._TP_KINDS or (self.ep is not None and kind in ("s13", "s2")):
            return None
        f, H, D = self.full_cfg, self.full_cfg.hidden_size, self.full_cfg.head_dim
        if kind == "lm_head":
            return None if self._vslice[2] == f.vocab_size else (f.vocab_size, H)
        return {"qkv": (f.q_size + 2 * f.kv_size, H), "qkv_bias": (f.q_size + 2 * f.kv_size,), "o": (H, f.q_size),
                "s13": (2 * f.shared_expert_intermediate_size, H), "s2": (H, f.shared_expert_intermediate_size),
                "mlp13": (2 * f.intermediate_size, H), "mlp2": (H, f.intermediate_size)}[kind]

    def shard(self, kind: str, full: torch.Tensor) -> torch.Tensor:
        """This rank's slice of an unsharded tensor (identity without TP): QKV rows of
        the local heads, o_proj columns, gate/up rows and down columns of the MLPs."""
        if self.tp is None or kind not in self._TP_KINDS or (self.ep is not None and kind in ("s13", "s2")):
            return full
        f, D = self.full_cfg, self.full_cfg.head_dim
        qh, kvh = self._tp_split
        r, w = self.tp.rank, self.tp.world
        if kind == "lm_head":
            v0, vl, width = self._vslice
            if width == full.shape[0]:
                return full
            out = full.new_zeros(width, full.shape[1])
            out[:vl] = full[v0:v0 + vl]
            return out
        if kind in ("qkv", "qkv_bias"):
            q = full[qh.start * D:qh.stop * D]
            k = full[f.q_size + kvh.start * D:f.q_size + kvh.stop * D]
            v = full[f.q_size + f.kv_size + kvh.start * D:f.q_size + f.kv_size + kvh.stop * D]
            return torch.cat([q, k, v], 0)
        if kind == "o":
            return full[:, qh.start * D:qh.stop * D]
        if kind in ("s13", "mlp13"):
            i = full.shape[0] // 2
            n = i // w
            return torch.cat([full[r * n:(r + 1) * n], full[i + r * n:i + (r + 1) * n]], 0)
        n = full.shape[1] // w
        return full[:, r * n:(r + 1) * n]

    @property
    def head_weight(self):
        """LM-head rows of this rank (the vocabulary slice under vocab-parallel TP)."""
        if self.lm_head is not None:
            return self.lm_head
        v0, vl, width = self._vslice
        return self.embed if vl == self.cfg.vocab_size else self.embed[v0:v0 + vl]

    # ------------------------------------------------------------------ workspaces
    def ensure_workspaces(self, max_tokens: int, max_batch: int, max_context: int):
        """Grow the MoE / decode scratch to cover these sizes.

        A replaced workspace is kept alive (``_retired_ws``): CUDA graphs that
        were captured with it still read and write its memory on replay."""
        cfg, dev = self.cfg, self.embed.device
        if cfg.num_experts and self.ep is None and (self._moe_ws is None or self._moe_ws.max_tokens < max_tokens):
            if self._moe_ws is not None:
                self._retired_ws.append(self._moe_ws)
            self._moe_ws = MoEWorkspace(max_tokens, cfg.num_experts, cfg.topk, cfg.hidden_size,
                                        cfg.moe_intermediate_size, dev, cfg.dtype)
        if dev.type == "cuda":
            ws = self._dec_ws
            need_splits = max(1, (max_context + 255) // 256)
            if ws is None or ws.max_splits < need_splits or ws.part_lse.numel() < max_batch * cfg.num_heads * need_splits:
                if ws is not None:
                    self._retired_ws.append(ws)
                self._dec_ws = DecodeWorkspace(max_batch, cfg.num_heads, cfg.head_dim, max_context, dev)

    # ------------------------------------------------------------------ forward
    def _mlp(self, L, x, i, norm=None):
        """MLP of layer i.  ``norm = (residual, next_weight, eps)`` (MoE layers only): the
        combine also does the next block's residual add + RMSNorm and returns its output."""
        cfg = self.cfg
        if cfg.is_moe_layer(i):
            shared_out = shared_gate = None
            if cfg.shared_expert_intermediate_size:
                shared_out = ops.linear(ops.linear(x, L.s13, gated=True), L.s2)
                if cfg.shared_expert_gate:
                    shared_gate = ops.linear(x, L.sgate, out_dtype=torch.float32)
            if self.ep is not None:
                return self.ep.forward(x, L.router, L.w13, L.w2, renormalize=cfg.norm_topk_prob,
                                       mode=cfg.router_mode, bias=getattr(L, "router_bias", None),
                                       n_group=cfg.n_group, topk_group=cfg.topk_group,
                                       scaling=cfg.routed_scaling_factor, shared_out=shared_out,
                                       shared_gate=shared_gate, norm=norm)
            if self._moe_ws is None:
                self.ensure_workspaces(max(x.shape[0], 4096), 1, 64)
            ws = self._moe_ws
            T, step = x.shape[0], ws.max_tokens
            if T <= step:
                return ops.fused_moe(x, L.router, L.w13, L.w2, cfg.topk, ws, renormalize=cfg.norm_topk_prob,
                                     mode=cfg.router_mode, bias=getattr(L, "router_bias", None), n_group=cfg.n_group,
                                     topk_group=cfg.topk_group, scaling=cfg.routed_scaling_factor,
                                     shared_out=shared_out, shared_gate=shared_gate, norm=norm)
            # more tokens than the (graph-captured) workspace holds: run in chunks
            out = torch.empty_like(x)
            for a in range(0, T, step):
                b = min(T, a + step)
                ops.fused_moe(x[a:b], L.router, L.w13, L.w2, cfg.topk, ws, renormalize=cfg.norm_topk_prob,
                              mode=cfg.router_mode, bias=getattr(L, "router_bias", None), n_group=cfg.n_group,
                              topk_group=cfg.topk_group, scaling=cfg.routed_scaling_factor, out=out[a:b],
                              shared_out=None if shared_out is None else shared_out[a:b],
                              shared_gate=None if shared_gate is None else shared_gate[a:b],
                              norm=None if norm is None else (norm[0][a:b], norm[1], norm[2]))
            return out
        return ops.linear(ops.linear(x, L.mlp13, gated=True), L.mlp2)

    def forward(self, fb: ForwardBatch, kv_cache: torch.Tensor) -> torch.Tensor:
        """Returns final-normed hidden states of ``fb.logits_indices`` rows (all rows if None).

        kv_cache: [layers, 2, pages, Hkv, 64, D].
        """
        if not self.embed.is_cuda:
            return self._forward(fb, kv_cache)
        with static_weights():  # the parameters are never written while a forward runs
            return self._forward(fb, kv_cache)

    def _forward(self, fb: ForwardBatch, kv_cache: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        if fb.input_embeds is not None:
            x = fb.input_embeds
        else:
            x = ops.embed(fb.input_ids, self.embed, fb.mm_index, fb.mm_embeds)
        T = x.shape[0]
        res = x.clone() if fb.input_embeds is not None else x
        if self.tp is not None:
            return self._forward_tp(fb, kv_cache, res)
        h = None
        fused_next = None    # this layer's input norm, already done by the previous MoE combine
        rot = cfg.rotary_dim or cfg.head_dim
        scale = 1.0 / math.sqrt(cfg.head_dim)
        nl = len(self.layers)
        for i, L in enumerate(self.layers):
            if fused_next is not None:
                normed, fused_next = fused_next, None
            elif h is None:
                normed = ops.rms_norm(res, L.ln1, cfg.rms_norm_eps)
            else:
                normed = ops.rms_norm(h, L.ln1, cfg.rms_norm_eps, residual=res)
            if i in fb.capture_layers:
                fb.captured[i] = res.clone()
            qkv = ops.linear(normed, L.qkv, bias=getattr(L, "qkv_bias", None))
            ops.qkv_rope_store(qkv, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, fb.positions, self.cos_tab,
                               self.sin_tab, rot, getattr(L, "q_norm", None), getattr(L, "k_norm", None),
                               cfg.rms_norm_eps, cfg.rope_neox, cfg.mrope_section, cfg.mrope_interleaved,
                               fb.slot_mapping, kv_cache[i, 0], kv_cache[i, 1])
            if fb.is_decode:
                attn = ops.decode_attention(qkv, kv_cache[i, 0], kv_cache[i, 1], fb.block_table, fb.kv_lens,
                                            cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, self._dec_ws, scale)
            else:
                attn = ops.prefill_attention(qkv, kv_cache[i, 0], kv_cache[i, 1], fb.block_table, fb.cu_q,
                                             fb.kv_lens, fb.tile_req, fb.tile_tok0, cfg.num_heads,
                                             cfg.num_kv_heads, cfg.head_dim, scale, tile_rows=fb.tile_rows)
            o = ops.linear(attn, L.o)
            normed2 = ops.rms_norm(o, L.ln2, cfg.rms_norm_eps, residual=res)
            has_ds = fb.deepstack is not None and i < len(fb.deepstack) and fb.deepstack[i] is not None
            if i + 1 < nl and cfg.is_moe_layer(i) and not has_ds:
                fused_next = self._mlp(L, normed2, i, norm=(res, self.layers[i + 1].ln1, cfg.rms_norm_eps))
                continue
            h = self._mlp(L, normed2, i)
            if has_ds:
                pos, emb = fb.deepstack[i]
                h.index_add_(0, pos, emb.to(h.dtype))
        if cfg.num_layers in fb.capture_layers:
            fb.captured[cfg.num_layers] = (res + h).clone()
        if fb.logits_indices is not None:
            sel = fb.logits_indices.long()
            return ops.rms_norm(h[sel], self.final_norm, cfg.rms_norm_eps, residual=res[sel].clone())
        return ops.rms_norm(h, self.final_norm, cfg.rms_norm_eps, residual=res)

    def _attention(self, L, i, normed, fb, kv_cache, wait=None):
        cfg = self.cfg
        qkv = ops.linear(normed, L.qkv, bias=getattr(L, "qkv_bias", None), wait=wait)
        ops.qkv_rope_store(qkv, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, fb.positions, self.cos_tab,
                           self.sin_tab, cfg.rotary_dim or cfg.head_dim, getattr(L, "q_norm", None),
                           getattr(L, "k_norm", None), cfg.rms_norm_eps, cfg.rope_neox, cfg.mrope_section,
                           cfg.mrope_interleaved, fb.slot_mapping, kv_cache[i, 0], kv_cache[i, 1])
        scale = 1.0 / math.sqrt(cfg.head_dim)
        if fb.is_decode:
            return ops.decode_attention(qkv, kv_cache[i, 0], kv_cache[i, 1], fb.block_table, fb.kv_lens,
                                        cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, self._dec_ws, scale)
        return ops.prefill_attention(qkv, kv_cache[i, 0], kv_cache[i, 1], fb.block_table, fb.cu_q, fb.kv_lens,
                                     fb.tile_req, fb.tile_tok0, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, scale,
                                     tile_rows=fb.tile_rows)

    def _forward_tp(self, fb: ForwardBatch, kv_cache: torch.Tensor, res: torch.Tensor) -> torch.Tensor:
        """Tensor-parallel forward: local heads / experts / MLP slices, every reduce point
        one fused kernel (owner scatter in the producer, reduce + residual + RMSNorm +
        all-gather in ``tp.reduce_norm``), the consumer GEMMs wait on the gather flags."""
        cfg, tp = self.cfg, self.tp
        T = res.shape[0]
        eps = cfg.rms_norm_eps
        nl = len(self.layers)
        if not res.is_cuda:
            raise RuntimeError("tensor parallelism runs on CUDA devices only")
        scatter = tp.scatter(T)
        normed, wait = ops.rms_norm(res, self.layers[0].ln1, eps), None
        if 0 in fb.capture_layers:
            fb.captured[0] = res.clone()
        for i, L in enumerate(self.layers):
            attn = self._attention(L, i, normed, fb, kv_cache, wait)
            ops.linear(attn, L.o, out=tp.part_local[:T], scatter=scatter)
            ep_layer = self.ep is not None and cfg.is_moe_layer(i)
            normed2 = tp.reduce_norm(res, L.ln2, eps, T, local_only=ep_layer)
            if ep_layer:
                self._moe_tp_ep(L, normed2, T)
            else:
                self._mlp_tp(L, normed2, i, T, scatter)
            if fb.deepstack is not None and i < len(fb.deepstack) and fb.deepstack[i] is not None:
                # deep-stack visual rows join the block output: the owner of each row adds them to
                # its residual rows before the reduce point sums the partials into them (the
                # other rows of `res` are not this rank's and are never read)
                pos, emb = fb.deepstack[i]
                res.index_add_(0, pos, emb.to(res.dtype))
            last = i + 1 == nl
            cap = (i + 1) in fb.capture_layers
            normed = tp.reduce_norm(res, self.final_norm if last else self.layers[i + 1].ln1, eps, T,
                                    gather_residual=cap, single_src=ep_layer)
            wait = tp.wait
            if cap:
                tp.wait_gather()
                fb.captured[i + 1] = tp.gres[:T].clone()
        tp.wait_gather()
        if fb.logits_indices is not None:
            return normed[fb.logits_indices.long()]
        return normed.clone()

    def _moe_tp_ep(self, L, x, T):
        """Expert-parallel MoE of the rows this TP rank owns (normalised in ``x[owned]`` by a
        local-only reduce point); the combined rows land in this rank's partial slot."""
        cfg, tp = self.cfg, self.tp
        a, b = tp.owned(T)
        xo = x[a:b]
        shared_out = shared_gate = None
        if cfg.shared_expert_intermediate_size and b > a:
            shared_out = ops.linear(ops.linear(xo, L.s13, gated=True), L.s2)
            if cfg.shared_expert_gate:
                shared_gate = ops.linear(xo, L.sgate, out_dtype=torch.float32)
        self.ep.forward(xo, L.router, L.w13, L.w2, renormalize=cfg.norm_topk_prob, mode=cfg.router_mode,
                        bias=getattr(L, "router_bias", None), n_group=cfg.n_group, topk_group=cfg.topk_group,
                        scaling=cfg.routed_scaling_factor, shared_out=shared_out, shared_gate=shared_gate,
                        out=tp.part_local[a:b])

    def _mlp_tp(self, L, x, i, T, scatter):
        """MLP of layer i on the gathered rows ``x``; writes this rank's partial rows to their owners."""
        cfg, tp = self.cfg, self.tp
        if not cfg.is_moe_layer(i):
            ops.linear(ops.linear(x, L.mlp13, gated=True, wait=tp.wait), L.mlp2, out=tp.part_local[:T],
                       scatter=scatter)
            return
        if self._moe_ws is None or self._moe_ws.max_tokens < T:
            self.ensure_workspaces(max(T, 4096), 1, 64)
        ws = self._moe_ws
        shared_out = shared_gate = None
        if cfg.shared_expert_intermediate_size:
            shared_out = ops.linear(ops.linear(x, L.s13, gated=True, wait=tp.wait), L.s2)
            if cfg.shared_expert_gate:
                shared_gate = ops.linear(x, L.sgate, out_dtype=torch.float32, wait=tp.wait)
        ops.tp_moe(x, L.router, L.w13, L.w2, cfg.topk, ws, self.expert0, tp, scatter,
                   renormalize=cfg.norm_topk_prob, mode=cfg.router_mode, bias=getattr(L, "router_bias", None),
                   n_group=cfg.n_group, topk_group=cfg.topk_group, scaling=cfg.routed_scaling_factor,
                   shared_out=shared_out, shared_gate=shared_gate)

    @torch.no_grad()
    def ep_idle(self):
        """An expert-parallel rank with no tokens this iteration: the MoE exchange of every layer
        with zero rows (its experts still serve the rows the other ranks dispatch)."""
        assert self.ep is not None, "idle forward of an expert-parallel model"
        cfg = self.cfg
        x = torch.empty(0, cfg.hidden_size, dtype=cfg.dtype, device=self.embed.device)
        for i, L in enumerate(self.layers):
            if cfg.is_moe_layer(i):
                self.ep.forward(x, L.router, L.w13, L.w2, renormalize=cfg.norm_topk_prob, mode=cfg.router_mode,
                                bias=getattr(L, "router_bias", None), n_group=cfg.n_group, topk_group=cfg.topk_group,
                                scaling=cfg.routed_scaling_factor)

    def close_parallel(self):
        """Collective: releases the peer-memory buffers of the TP / EP exchange."""
        if self.vocab_sampler is not None:
            self.vocab_sampler.close()
            self.vocab_sampler = None
        for par in (self.tp, self.ep):
            if par is not None:
                par.close()

    def local_logits(self, hidden: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """fp32 logits of this rank's LM-head rows (all of them without vocab-parallel TP)."""
        if not hidden.is_cuda:
            return ops.linear(hidden, self.head_weight, out=out, out_dtype=torch.float32)
        with static_weights():
            return ops.linear(hidden, self.head_weight, out=out, out_dtype=torch.float32)

    def logits(self, hidden: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Full-vocabulary fp32 logits.  Under vocab-parallel TP the slices are all-gathered
        with torch.distributed (a process group must be initialised); the serving path
        never calls this, it draws tokens with :meth:`sample_tokens`."""
        if self.vocab_sampler is None:
            return self.local_logits(hidden, out)
        import torch.distributed as dist

        loc = self.local_logits(hidden)
        parts = [torch.empty_like(loc) for _ in range(self.tp.world)]
        dist.all_gather(parts, loc.contiguous())
        full = torch.cat(parts, 1)[:, :self.full_cfg.vocab_size]
        if out is not None:
            out.copy_(full)
            return out
        return full

    def sample_tokens(self, hidden: torch.Tensor, st=None, suppress=(-1, -1, -1), out: torch.Tensor | None = None,
                      row_slot: torch.Tensor | None = None, slot_tokens: torch.Tensor | None = None) -> torch.Tensor:
        """LM head + sampling: int32 tokens [rows] (identical on every TP rank)."""
        from ..ops.sampling import sample

        if self.vocab_sampler is None:
            return sample(self.local_logits(hidden), st, suppress, out=out, row_slot=row_slot,
                          slot_tokens=slot_tokens)
        return self.vocab_sampler.sample(self.local_logits(hidden), st, suppress, out=out, row_slot=row_slot,
                                         slot_tokens=slot_tokens)
