"""Ming-Omni talker: a dense Qwen2 LM that generates continuous audio latents.

Per generated patch (``patch_size`` latent frames of ``latent_dim``):

1. the LM's last hidden state conditions a flow-matching sampler (CFM): a
   bidirectional transformer ("DiT") over [t + cond token, 32 history patches,
   current patch] predicts a velocity; ``steps`` Euler steps along the
   sway-warped EPSS schedule with classifier-free guidance (conditional and
   null-condition rows in one batch) turn Gaussian noise into the patch;
2. an aggregator transformer folds the patch into one LM input embedding (a cls
   row), which is the LM's next input;
3. a linear stop head on the LM hidden state gives the end-of-speech probability.

This build batches every concurrent stream in lock step and captures one whole
step (LM decode, all CFM steps, aggregator, stop head) as ONE CUDA graph per
batch bucket; every projection is the tcgen05 GEMM, the attention is the
ragged non-causal attention kernel (rows of a stream attend only to that
stream's tokens), the norms are the RMSNorm kernel and the rotary embedding is
the interleaved-pair mode of the fused QK-RoPE kernel.  Head sizes the kernels
do not take (72 for a 1152-wide aggregator with 16 heads) are zero-padded per
head (with the attention scale of the true size), which leaves the math unchanged.

Reference counterparts: MingOmniTalker.generate / CFMGraphExecutor
(sglang_omni/models/ming_omni/talker/modeling_ming_omni_talker.py:93-183,408-563),
CFM.sample and the EPSS timesteps (talker/talker_module/cfm.py:8-60), DiT and its
embedders (talker/talker_module/dit.py:22-208), Aggregator
(talker/talker_module/aggregator.py:19-86), DiTBlock / Attention / FinalLayer
(talker/talker_module/modules.py:25-283), the prompt layout of
omni_audio_generation_func (modeling_ming_omni_talker.py:565-672).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch
from torch import nn

from ... import ops
from ...engines.ar.kv_pool import KVPool
from ...environ import environ
from ...ops.gemm import static_weights
from ...utils.cuda_graph import capture_graph
from ...utils.hostdev import h2d
from ..decoder import DecoderConfig, DecoderLM, ForwardBatch

# Euler step grids of the CFM sampler, in units of 1/32 (EPSS schedules)
_EPSS = {5: [0, 2, 4, 8, 16, 32], 6: [0, 2, 4, 6, 8, 16, 32], 7: [0, 2, 4, 6, 8, 16, 24, 32],
         10: [0, 2, 4, 6, 8, 12, 16, 20, 24, 28, 32], 12: [0, 2, 4, 6, 8, 10, 12, 14, 16, 20, 24, 28, 32],
         16: [0, 1, 2, 3, 4, 5, 6, 7, 8, 10, 12, 14, 16, 20, 24, 28, 32]}


def cfm_timesteps(steps: int, sway: float | None = -1.0) -> list[float]:
    """EPSS grid (uniform when no table exists) warped by sway sampling
    t + s (cos(pi t / 2) - 1 + t)."""
    if steps in _EPSS:
        t = [v / 32.0 for v in _EPSS[steps]]
    else:
        t = [i / steps for i in range(steps + 1)]
    if sway is not None:
        t = [v + sway * (math.cos(math.pi / 2 * v) - 1 + v) for v in t]
    return t


def qwen2_config(**over) -> DecoderConfig:
    """The talker LM (Qwen2-0.5B layout: 24 layers, hidden 896, 14 / 2 heads of 64, q/k/v biases)."""
    c = DecoderConfig(vocab_size=151936, hidden_size=896, num_layers=24, num_heads=14, num_kv_heads=2, head_dim=64,
                      intermediate_size=4864, rope_theta=1e6, qk_norm=False, attention_bias=True,
                      tie_word_embeddings=True, rms_norm_eps=1e-6, max_position=32768, name="ming_talker_llm")
    for k, v in over.items():
        setattr(c, k, v)
    return c


@dataclass
class MingTalkerConfig:
    llm: DecoderConfig = field(default_factory=qwen2_config)
    dit_hidden: int = 1024
    dit_depth: int = 28
    dit_heads: int = 16
    dit_mlp_ratio: float = 4.0
    agg_hidden: int = 1152
    agg_depth: int = 28
    agg_heads: int = 16
    agg_mlp_ratio: float = 4.0
    patch_size: int = 4
    history_patch_size: int = 32
    latent_dim: int = 64
    spk_dim: int = 192
    steps: int = 10
    freq_embed_dim: int = 256
    dtype: torch.dtype = torch.bfloat16

    @classmethod
    def from_dict(cls, raw: dict, llm: dict | None = None) -> "MingTalkerConfig":
        """From the checkpoint's config.json (``flowmodel`` / ``aggregator`` sub-dicts) and llm/config.json."""
        fm, ag = raw.get("flowmodel", {}) or {}, raw.get("aggregator", {}) or {}
        lc = llm or {}
        heads = lc.get("num_attention_heads", 14)
        hidden = lc.get("hidden_size", 896)
        lm = qwen2_config(vocab_size=lc.get("vocab_size", 151936), hidden_size=hidden,
                          num_layers=lc.get("num_hidden_layers", 24), num_heads=heads,
                          num_kv_heads=lc.get("num_key_value_heads", 2), head_dim=hidden // heads,
                          intermediate_size=lc.get("intermediate_size", 4864), rope_theta=lc.get("rope_theta", 1e6),
                          rms_norm_eps=lc.get("rms_norm_eps", 1e-6),
                          tie_word_embeddings=lc.get("tie_word_embeddings", True))
        return cls(llm=lm, dit_hidden=fm.get("hidden_size", 1024), dit_depth=fm.get("depth", 28),
                   dit_heads=fm.get("num_heads", 16), dit_mlp_ratio=fm.get("mlp_ratio", 4.0),
                   agg_hidden=ag.get("hidden_size", 1152), agg_depth=ag.get("depth", 28),
                   agg_heads=ag.get("num_heads", 16), agg_mlp_ratio=ag.get("mlp_ratio", 4.0),
                   patch_size=raw.get("patch_size", 4), history_patch_size=raw.get("history_patch_size", 32),
                   latent_dim=raw.get("latent_dim", 64), spk_dim=raw.get("spk_dim", 192),
                   steps=raw.get("steps", 10))


def _kernel_head_dim(d: int) -> int:
    """Smallest head size both the QK-RoPE and the attention kernels take."""
    for k in (64, 96, 128):
        if d <= k:
            return k
    raise ValueError(f"head size {d} > 128")


class BlockStack(nn.Module):
    """Pre-norm bidirectional transformer blocks (RMSNorm, q/k/v/o with biases,
    interleaved-pair RoPE over each stream's positions, GELU-tanh MLP) on the
    kernels, over ragged per-stream sequences.  The weights keep the q/k/v
    projections fused per layer ([3 * heads * Dk, hidden], head-padded to the
    kernel head size Dk)."""

    def __init__(self, hidden: int, depth: int, heads: int, mlp_ratio: float, device, dtype):
        super().__init__()
        self.hidden, self.depth, self.heads = hidden, depth, heads
        self.d = hidden // heads
        self.dk = _kernel_head_dim(self.d)
        self.inner = int(hidden * mlp_ratio)
        P = lambda *s: nn.Parameter(torch.empty(*s, dtype=dtype, device=device), requires_grad=False)  # noqa: E731
        self.layers = nn.ModuleList()
        for _ in range(depth):
            L = nn.Module()
            L.n1, L.n2 = P(hidden), P(hidden)
            L.qkv, L.qkv_b = P(3 * heads * self.dk, hidden), P(3 * heads * self.dk)
            L.o, L.o_b = P(hidden, heads * self.dk), P(hidden)
            L.f1, L.f1_b = P(self.inner, hidden), P(self.inner)
            L.f2, L.f2_b = P(hidden, self.inner), P(hidden)
            self.layers.append(L)
        self.max_pos = 4096
        cos, sin = ops.rope_tables(self.d, 10000.0, self.max_pos, device, round_bf16=False)
        self.register_buffer("cos", cos, persistent=False)
        self.register_buffer("sin", sin, persistent=False)

    # -------------------------------------------------------------- weights
    def pad_heads(self, w: torch.Tensor) -> torch.Tensor:
        """[heads * d, ...] -> [heads * dk, ...] with zero rows for the padding of every head."""
        if self.dk == self.d:
            return w
        shp = w.shape
        out = w.new_zeros((self.heads, self.dk) + tuple(shp[1:]))
        out[:, : self.d] = w.reshape((self.heads, self.d) + tuple(shp[1:]))
        return out.reshape((self.heads * self.dk,) + tuple(shp[1:]))

    def set_layer(self, i: int, sd: dict[str, torch.Tensor], prefix: str):
        """From the reference layout (``norm1``, ``attn.to_q/to_k/to_v/to_out.0``, ``mlp.ff.0.0``, ``mlp.ff.2``)."""
        L = self.layers[i]
        g = lambda k: sd[prefix + k]  # noqa: E731
        L.n1.copy_(g("norm1.weight"))
        L.n2.copy_(g("norm2.weight"))
        L.qkv.copy_(torch.cat([self.pad_heads(g(f"attn.to_{n}.weight")) for n in "qkv"], 0))
        L.qkv_b.copy_(torch.cat([self.pad_heads(g(f"attn.to_{n}.bias")) for n in "qkv"], 0))
        o = g("attn.to_out.0.weight")
        if self.dk != self.d:
            o = self.pad_heads(o.t().contiguous()).t()
        L.o.copy_(o)
        L.o_b.copy_(g("attn.to_out.0.bias"))
        L.f1.copy_(g("mlp.ff.0.0.weight"))
        L.f1_b.copy_(g("mlp.ff.0.0.bias"))
        L.f2.copy_(g("mlp.ff.2.weight"))
        L.f2_b.copy_(g("mlp.ff.2.bias"))

    def random_init_(self, gen: torch.Generator, std: float):
        for L in self.layers:
            L.n1.fill_(1.0)
            L.n2.fill_(1.0)
            for name in ("qkv", "o", "f1", "f2"):
                w = getattr(L, name)
                w.copy_((torch.randn(w.shape, generator=gen) * std).to(w.dtype))
            for name in ("qkv_b", "o_b", "f1_b", "f2_b"):
                b = getattr(L, name)
                b.copy_((torch.randn(b.shape, generator=gen) * std).to(b.dtype))
            if self.dk != self.d:  # keep the padding rows / columns zero
                D, dk, h = self.d, self.dk, self.heads
                L.qkv.view(3, h, dk, -1)[:, :, D:] = 0
                L.qkv_b.view(3, h, dk)[:, :, D:] = 0
                L.o.view(self.hidden, h, dk)[:, :, D:] = 0

    # -------------------------------------------------------------- forward
    def forward(self, x: torch.Tensor, positions: torch.Tensor, cu: torch.Tensor, q_lens: list[int],
                tiles=None) -> torch.Tensor:
        """x: [T, hidden] rows of all streams; positions: int32 [T] (position inside its stream);
        cu: int32 [B + 1] stream row offsets."""
        h, d, dk = self.heads, self.d, self.dk
        scale = 1.0 / math.sqrt(d)
        for L in self.layers:
            n = ops.rms_norm(x, L.n1, 1e-6)
            qkv = ops.linear(n, L.qkv, bias=L.qkv_b)
            ops.qkv_rope_store(qkv, h, h, dk, positions, self.cos, self.sin, rot_dim=d, neox=False)
            q, k, v = qkv.split(h * dk, dim=1)
            a = ops.varlen_attention(q, k, v, cu, h, h, dk, scale=scale, causal=False, q_lens=q_lens, tiles=tiles)
            x = ops.linear(a, L.o, bias=L.o_b, residual=x)
            n = ops.rms_norm(x, L.n2, 1e-6)
            f = ops.linear(n, L.f1, bias=L.f1_b, act="gelu_tanh")
            x = ops.linear(f, L.f2, bias=L.f2_b, residual=x)
        return x


def timestep_embedding(t: torch.Tensor, dim: int, scale: float = 1000.0) -> torch.Tensor:
    """Sinusoidal embedding [sin(s t w_i), cos(s t w_i)], w_i = 10000^(-i / (dim/2 - 1))."""
    half = dim // 2
    w = torch.exp(torch.arange(half, device=t.device, dtype=torch.float32) * -(math.log(10000.0) / (half - 1)))
    e = scale * t.float()[:, None] * w[None, :]
    return torch.cat([e.sin(), e.cos()], dim=-1)


class MingTalker(nn.Module):
    def __init__(self, cfg: MingTalkerConfig = MingTalkerConfig(), device="cpu"):
        super().__init__()
        self.cfg = cfg
        dt = cfg.dtype
        self.lm = DecoderLM(cfg.llm, device=device)
        H, Dd, Da, Z = cfg.llm.hidden_size, cfg.dit_hidden, cfg.agg_hidden, cfg.latent_dim
        P = lambda *s: nn.Parameter(torch.empty(*s, dtype=dt, device=device), requires_grad=False)  # noqa: E731
        # DiT embedders and head
        self.t1, self.t1_b = P(Dd, cfg.freq_embed_dim), P(Dd)
        self.t2, self.t2_b = P(Dd, Dd), P(Dd)
        self.x_emb, self.x_emb_b = P(Dd, Z), P(Dd)
        self.c_emb, self.c_emb_b = P(Dd, H), P(Dd)
        self.spk_emb, self.spk_emb_b = P(Dd, cfg.spk_dim), P(Dd)
        self.dit = BlockStack(Dd, cfg.dit_depth, cfg.dit_heads, cfg.dit_mlp_ratio, device, dt)
        self.dit_norm = P(Dd)
        self.dit_out, self.dit_out_b = P(Z, Dd), P(Z)
        # aggregator
        self.a_x, self.a_x_b = P(Da, Z), P(Da)
        self.a_cls = P(Da)
        self.agg = BlockStack(Da, cfg.agg_depth, cfg.agg_heads, cfg.agg_mlp_ratio, device, dt)
        self.agg_norm = P(Da)
        self.agg_out, self.agg_out_b = P(H, Da), P(H)
        # stop head and speaker projection into the LM
        self.stop, self.stop_b = P(2, H), P(2)
        self.spk_head, self.spk_head_b = P(H, cfg.spk_dim), P(H)

    @property
    def device(self):
        return self.stop.device

    def random_init_(self, seed: int = 0, std: float = 0.02):
        self.lm.random_init_(seed=seed, std=std)
        g = torch.Generator().manual_seed(seed + 17)
        for name, p in self.named_parameters():
            if name.startswith(("lm.", "dit.", "agg.")):
                continue
            if name.endswith("norm"):
                p.fill_(1.0)
            else:
                p.copy_((torch.randn(p.shape, generator=g) * std).to(p.dtype))
        self.dit.random_init_(g, std)
        self.agg.random_init_(g, std)
        return self

    def load_state_dict_ref(self, sd: dict[str, torch.Tensor]):
        """From the reference checkpoint layout (``model.*`` Qwen2, ``cfm.model.*`` DiT,
        ``aggregator.*``, ``stop_head``, ``spk_head``)."""
        from ..weight_loader import load_decoder_from_hf

        load_decoder_from_hf(self.lm, sd, "model.")
        d = "cfm.model."
        pairs = [("t1", d + "t_embedder.time_mlp.0"), ("t2", d + "t_embedder.time_mlp.2"), ("x_emb", d + "x_embedder"),
                 ("c_emb", d + "c_embedder.cond_embedder"), ("dit_out", d + "final_layer.linear"),
                 ("a_x", "aggregator.x_embedder"), ("agg_out", "aggregator.final_layer.linear"),
                 ("stop", "stop_head"), ("spk_head", "spk_head")]
        if d + "spk_embedder.weight" in sd:
            pairs.append(("spk_emb", d + "spk_embedder"))
        for ours, theirs in pairs:
            getattr(self, ours).copy_(sd[theirs + ".weight"])
            getattr(self, ours + "_b").copy_(sd[theirs + ".bias"])
        self.dit_norm.copy_(sd[d + "final_layer.norm_final.weight"])
        self.agg_norm.copy_(sd["aggregator.final_layer.norm_final.weight"])
        self.a_cls.copy_(sd["aggregator.word_embedder.weight"][0])
        for i in range(self.cfg.dit_depth):
            self.dit.set_layer(i, sd, f"{d}blocks.{i}.")
        for i in range(self.cfg.agg_depth):
            self.agg.set_layer(i, sd, f"aggregator.blocks.{i}.")

    # -------------------------------------------------------------- building blocks
    def dit_velocity(self, x: torch.Tensor, t: torch.Tensor, cond: torch.Tensor, his: torch.Tensor,
                     rows: "RowLayout") -> torch.Tensor:
        """Velocity of the current patch. x [N, P, Z], t [N] (fp32), cond [N, H] (zeros for the
        null rows of classifier-free guidance), his [N, Hp, Z] -> [N, P, Z]."""
        N, Pn, Z = x.shape
        te = timestep_embedding(t, self.cfg.freq_embed_dim).to(self.cfg.dtype)
        te = ops.linear(ops.linear(te, self.t1, bias=self.t1_b, act="silu"), self.t2, bias=self.t2_b)
        y = ops.linear(cond, self.c_emb, bias=self.c_emb_b, residual=te)            # [N, Dd] = t + c
        lat = ops.linear(torch.cat([his, x], 1).reshape(-1, Z), self.x_emb, bias=self.x_emb_b)
        seq = torch.cat([y.unsqueeze(1), lat.view(N, -1, lat.shape[-1])], 1).reshape(-1, lat.shape[-1])
        h = self.dit(seq, rows.pos, rows.cu, rows.lens, rows.tiles)
        h = h.view(N, -1, h.shape[-1])[:, -Pn:].reshape(-1, h.shape[-1])
        out = ops.linear(ops.rms_norm(h, self.dit_norm, 1e-6), self.dit_out, bias=self.dit_out_b)
        return out.view(N, Pn, Z)

    def cfm_sample(self, cond: torch.Tensor, his: torch.Tensor, noise: torch.Tensor, ts: list[float],
                   cfg_strength: float, rows: "RowLayout") -> torch.Tensor:
        """Euler integration of the guided velocity from noise [B, P, Z] at t=0 to t=1."""
        B = cond.shape[0]
        cond2 = torch.cat([cond, torch.zeros_like(cond)], 0)
        his2 = torch.cat([his, his], 0)
        y = noise
        for s in range(len(ts) - 1):
            t = torch.full((2 * B,), ts[s], dtype=torch.float32, device=cond.device)
            v = self.dit_velocity(torch.cat([y, y], 0), t, cond2, his2, rows)
            vc, vn = v[:B].float(), v[B:].float()
            y = (y.float() + (vc + (vc - vn) * cfg_strength) * (ts[s + 1] - ts[s])).to(noise.dtype)
        return y

    def aggregate(self, lat: torch.Tensor, rows: "RowLayout") -> torch.Tensor:
        """[B, P, Z] patch -> [B, H] LM input embedding (the cls row of the aggregator)."""
        B, Pn, Z = lat.shape
        x = ops.linear(lat.reshape(-1, Z), self.a_x, bias=self.a_x_b).view(B, Pn, -1)
        seq = torch.cat([self.a_cls.view(1, 1, -1).expand(B, 1, -1), x], 1).reshape(B * (Pn + 1), -1)
        h = self.agg(seq, rows.pos, rows.cu, rows.lens, rows.tiles)
        cls = h.view(B, Pn + 1, -1)[:, 0]
        return ops.linear(ops.rms_norm(cls.contiguous(), self.agg_norm, 1e-6), self.agg_out, bias=self.agg_out_b)

    def stop_prob(self, hidden: torch.Tensor) -> torch.Tensor:
        lg = ops.linear(hidden, self.stop, bias=self.stop_b, out_dtype=torch.float32)
        return torch.softmax(lg, dim=-1)[:, 1]

    def project_speaker(self, spk: torch.Tensor) -> torch.Tensor:
        return ops.linear(spk.to(self.cfg.dtype).view(-1, self.cfg.spk_dim), self.spk_head, bias=self.spk_head_b)


class RowLayout:
    """Ragged layout of N equal-length sequences of L rows for the block stacks:
    positions 0..L-1 per sequence, row offsets, and the attention's tile table."""

    def __init__(self, n: int, length: int, device):
        self.n, self.length = n, length
        self.lens = [length] * n
        self.pos = torch.arange(length, dtype=torch.int32, device=device).repeat(n)
        self.cu = torch.arange(0, (n + 1) * length, length, dtype=torch.int32, device=device)
        self.tiles = None
        if torch.device(device).type == "cuda":
            req, tok0 = ops.prefill_tiles(self.lens, 1)
            self.tiles = (h2d(req, device, torch.int32), h2d(tok0, device, torch.int32))


@dataclass
class MingStream:
    rid: str
    slot: int
    max_patches: int
    min_patches: int = 3
    pages: list = field(default_factory=list)
    num_cached: int = 0
    patches: int = 0
    done: bool = False
    latents: list = field(default_factory=list)   # host [P, Z] float32 per generated patch


class MingSpeechGenerator:
    """All concurrent talker streams in lock step: one LM decode + CFM + aggregator +
    stop head per step for every stream (one CUDA graph per batch bucket)."""

    def __init__(self, talker: MingTalker, max_streams: int = 32, max_context: int = 1024, cfg_strength: float = 2.0,
                 stop_threshold: float = 0.5, use_graphs: bool = True, seed: int = 0):
        self.t = talker
        c = talker.cfg
        lc = c.llm
        dev = talker.device
        self.device = dev
        self.max_streams = max_streams
        self.max_pages = (max_context + 63) // 64
        self.pool = KVPool(lc.num_layers, lc.num_kv_heads, lc.head_dim, max_streams * self.max_pages + 2, dev, lc.dtype)
        talker.lm.ensure_workspaces(max(max_streams, 512) * 4, max_streams, max_context)
        S = max_streams + 1   # slot 0 = padding
        self.feedback = torch.zeros(S, lc.hidden_size, dtype=lc.dtype, device=dev)
        self.his = torch.zeros(S, c.history_patch_size, c.latent_dim, dtype=c.dtype, device=dev)
        self.lat_out = torch.zeros(S, c.patch_size, c.latent_dim, dtype=c.dtype, device=dev)
        self.stop_out = torch.zeros(S, dtype=torch.float32, device=dev)
        self.noise_step = torch.zeros(S, dtype=torch.int64, device=dev)
        self.noise_seed = int(seed)
        self.cfg_strength = cfg_strength
        self.stop_threshold = stop_threshold
        self.ts = cfm_timesteps(c.steps)
        self.streams: dict[str, MingStream] = {}
        self.free_slots = list(range(S - 1, 0, -1))
        self.use_graphs = use_graphs and dev.type == "cuda" and environ.OMNI_USE_CUDA_GRAPHS.get()
        self.graphs: dict[int, tuple] = {}
        self.buckets = [b for b in (1, 2, 4, 8, 16, 24, 32, 48, 64) if b <= max_streams]
        if self.buckets[-1] < max_streams:
            self.buckets.append(max_streams)
        self._layouts: dict[int, tuple] = {}
        PB = max_streams
        from ...utils.staging import PinnedRing

        self.meta_ring = PinnedRing(6 * PB + PB * self.max_pages, torch.int32, 2, dev.type == "cuda")
        self.meta_dev = torch.zeros(6 * PB + PB * self.max_pages, dtype=torch.int32, device=dev)
        from ... import _runtime as rt

        self.builder = rt.DecodeMetaBuilder(PB, self.max_pages)

    # ------------------------------------------------------------------ streams
    def add_stream(self, rid: str, prefill_embeds: torch.Tensor, prompt_latents: torch.Tensor | None = None,
                   max_patches: int = 256, min_patches: int = 3) -> MingStream:
        if not self.free_slots:
            raise RuntimeError("no free talker slots")
        slot = self.free_slots.pop()
        room = self.max_pages * 64 - prefill_embeds.shape[0]
        st = MingStream(rid, slot, max_patches=max(1, min(max_patches, room)), min_patches=min_patches)
        st._prefill = prefill_embeds
        self.his[slot].zero_()
        self.noise_step[slot] = 0
        if prompt_latents is not None:  # voice prompt: its last latent frames seed the history
            Hp = self.t.cfg.history_patch_size
            pl = prompt_latents.to(self.his.dtype).to(self.device)[-Hp:]
            self.his[slot, Hp - pl.shape[0]:] = pl
        self.streams[rid] = st
        return st

    def remove(self, rid: str):
        st = self.streams.pop(rid, None)
        if st is not None:
            self.pool.free(st.pages)
            st.pages = []
            self.free_slots.append(st.slot)

    def _layout(self, PB: int):
        lay = self._layouts.get(PB)
        if lay is None:
            c = self.t.cfg
            lay = (RowLayout(2 * PB, 1 + c.history_patch_size + c.patch_size, self.device),
                   RowLayout(PB, 1 + c.patch_size, self.device))
            self._layouts[PB] = lay
        return lay

    def _tail(self, hidden: torch.Tensor, slots: torch.Tensor, PB: int):
        """CFM + aggregator + stop head for the rows of `slots`; writes the slot state."""
        c = self.t.cfg
        sl = slots.long()
        dit_rows, agg_rows = self._layout(PB)
        noise = self._noise(sl).to(c.dtype)
        his = self.his[sl]
        lat = self.t.cfm_sample(hidden, his, noise, self.ts, self.cfg_strength, dit_rows)
        emb = self.t.aggregate(lat, agg_rows)
        stop = self.t.stop_prob(hidden)
        self.feedback[sl] = emb.to(self.feedback.dtype)
        self.his[sl] = torch.cat([his[:, c.patch_size:], lat], 1)
        self.lat_out[sl] = lat
        self.stop_out[sl] = stop

    def _noise(self, sl: torch.Tensor) -> torch.Tensor:
        """Gaussian start noise [n, P, Z] of each slot's next patch from a counter hash
        (slot, patch counter, element) and Box-Muller: no generator state, so the
        captured step draws fresh noise on every replay and threads never share a
        generator with another thread's graph capture."""
        c = self.t.cfg
        n = c.patch_size * c.latent_dim
        e = torch.arange(n, device=self.device, dtype=torch.int64)[None, :]
        base = sl[:, None] * 1000003 + self.noise_step[sl][:, None] * 7919 + self.noise_seed
        u1 = _hash_uniform(base * 2 * n + 2 * e)
        u2 = _hash_uniform(base * 2 * n + 2 * e + 1)
        self.noise_step[sl] += 1
        z = torch.sqrt(-2.0 * torch.log(u1)) * torch.cos(2 * math.pi * u2)
        return z.view(-1, c.patch_size, c.latent_dim)

    @torch.no_grad()
    def prefill(self, streams: list[MingStream]):
        if not streams:
            return
        dev = self.device
        lm = self.t.lm
        embeds = [s._prefill for s in streams]
        lens = [e.shape[0] for e in embeds]
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
        req, tok0 = ops.prefill_tiles(lens, lm.cfg.num_heads // lm.cfg.num_kv_heads)
        d = lambda a: h2d(a, dev)  # noqa: E731
        fb = ForwardBatch(is_decode=False, positions=d(np.stack([pos] * 3)), slot_mapping=d(slot_map),
                          kv_lens=h2d(lens, dev, torch.int32), block_table=d(bt),
                          input_embeds=torch.cat(embeds, 0).to(lm.cfg.dtype), cu_q=d(cu),
                          tile_req=h2d(req, dev, torch.int32), tile_tok0=h2d(tok0, dev, torch.int32),
                          logits_indices=d(cu[1:] - 1))
        hidden = lm(fb, self.pool.kv)
        slots = h2d([s.slot for s in streams], dev, torch.int32)
        PB = len(streams)
        with static_weights() if dev.type == "cuda" else _null():
            self._tail(hidden, slots, PB)
        for s, n in zip(streams, lens):
            s.num_cached = n
            del s._prefill
        self._collect(streams)

    def _views(self, PB):
        m = self.meta_dev
        P = self.max_pages
        return (m[0:PB], m[PB:2 * PB], m[2 * PB:5 * PB].view(3, PB), m[5 * PB:6 * PB],
                m[6 * PB:6 * PB + PB * P].view(PB, P))

    def _step_body(self, PB):
        kv_lens, slot_mapping, positions, slots, bt = self._views(PB)
        fb = ForwardBatch(is_decode=True, positions=positions, slot_mapping=slot_mapping, kv_lens=kv_lens,
                          block_table=bt, input_embeds=self.feedback[slots.long()])
        hidden = self.t.lm(fb, self.pool.kv)
        with static_weights() if self.device.type == "cuda" else _null():
            self._tail(hidden, slots, PB)
        return hidden

    def _bucket(self, n):
        for b in self.buckets:
            if b >= n:
                return b
        raise ValueError(n)

    def _fill_meta(self, streams, PB):
        host = self.meta_ring.next().numpy()
        B = len(streams)
        kl = np.fromiter((s.num_cached for s in streams), dtype=np.int64, count=B)
        md = np.zeros(B, dtype=np.int64)
        sl = np.fromiter((s.slot for s in streams), dtype=np.int64, count=B)
        self.builder.build(host, [s.pages for s in streams], kl, md, sl, self.pool.allocator_native(), PB)
        self.meta_ring.upload(self.meta_dev, 6 * PB + PB * self.max_pages)

    def _capture(self, PB):
        self._layout(PB)  # its host-to-device copies must not be part of the graph
        host = self.meta_ring.next().numpy()
        n = 6 * PB + PB * self.max_pages
        host[:n] = 0
        host[PB:2 * PB] = -1
        self.meta_ring.upload(self.meta_dev, n, blocking=True)
        saved = (self.feedback[0].clone(), self.his[0].clone(), self.noise_step.clone())
        g, _ = capture_graph(lambda: self._step_body(PB))
        self.feedback[0].copy_(saved[0])
        self.his[0].copy_(saved[1])
        self.noise_step.copy_(saved[2])
        self.graphs[PB] = g

    def capture_all(self):
        if self.use_graphs:
            for PB in self.buckets:
                if PB not in self.graphs:
                    self._capture(PB)

    @torch.no_grad()
    def step(self, streams: list[MingStream]):
        """One patch for every stream in `streams` (each already prefilled)."""
        B = len(streams)
        PB = self._bucket(B)
        if self.use_graphs and PB not in self.graphs:
            self._capture(PB)
        self._fill_meta(streams, PB)
        if self.use_graphs:
            self.graphs[PB].replay()
        else:
            self._step_body(PB)
        for s in streams:
            s.num_cached += 1
        self._collect(streams)

    def _collect(self, streams: list[MingStream]):
        idx = torch.tensor([s.slot for s in streams], dtype=torch.long, device=self.device)
        lat = self.lat_out[idx].float().cpu()
        stop = self.stop_out[idx].cpu()
        for i, s in enumerate(streams):
            s.latents.append(lat[i])
            s.patches += 1
            if (s.patches > s.min_patches and float(stop[i]) > self.stop_threshold) or s.patches >= s.max_patches:
                s.done = True

    def run(self, streams: list[MingStream]) -> None:
        """Prefills `streams` and steps all unfinished ones until every stream is done."""
        self.prefill([s for s in streams if hasattr(s, "_prefill")])
        while True:
            live = [s for s in streams if not s.done]
            if not live:
                return
            self.step(live)


def _mix64(z: torch.Tensor) -> torch.Tensor:
    """SplitMix64-style finaliser on int64 (wrapping multiplies; arithmetic shifts)."""
    z = (z ^ (z >> 30)) * -4658895280553007687     # 0xBF58476D1CE4E5B9 as a signed int64
    z = (z ^ (z >> 27)) * -7723592293110705685     # 0x94D049BB133111EB
    return z ^ (z >> 31)


def _hash_uniform(x: torch.Tensor) -> torch.Tensor:
    """Uniform in (0, 1) from bits 10..62 of the mixed counter (the last xor-shift
    leaves bit 63 clear with arithmetic shifts)."""
    z = _mix64(x * -7046029254386353131)           # 0x9E3779B97F4A7C15
    return (((z >> 10) & ((1 << 53) - 1)).double() + 0.5) / float(1 << 53)


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def build_talker_prompt(tok, text: str, prompt: str = "Please generate speech based on the following description.\n",
                        instruction: str | None = None, n_speakers: int = 0, n_prompt_latents: int = 0,
                        prompt_text: str | None = None) -> tuple[list[int], dict]:
    """Token ids of the talker prompt and the rows whose embeddings are replaced:
    ``spk`` rows (after each ``<|vision_start|>``) take projected speaker embeddings,
    ``latent`` rows (after ``<audio>``) take voice-prompt patch embeddings."""
    enc = lambda s: list(tok.encode(s))  # noqa: E731
    spk: list[int] = []
    for i in range(n_speakers):
        spk += enc(f"  speaker_{i + 1}:") + enc("<|vision_start|>") + enc("<|vision_pad|>") + enc("<|vision_end|>\n")
    instr = enc(instruction) + enc("<|im_end|>") if instruction else []
    ptxt, plat = [], []
    if n_prompt_latents and prompt_text is not None:
        ptxt = enc(prompt_text)
        plat = enc("<audioPatch>") * n_prompt_latents
    head = enc(" Text input:\n")
    if all(k in text for k in ("Genre: ", "Mood: ", "Instrument: ", "Theme: ", "Duration: ")):
        head = []
    ids = (enc("<|im_start|>system\nYou are a helpful assistant.<|im_end|>\n") + enc("<|im_start|>user\n")
           + enc(prompt) + spk + head + ptxt + enc(text) + enc("<|im_end|>\n") + enc("<|im_start|>assistant\n")
           + instr + enc("<audio>") + plat)
    vs = enc("<|vision_start|>")
    au = enc("<audio>")
    spk_rows = [i + 1 for i, t in enumerate(ids) if len(vs) == 1 and t == vs[0]][:n_speakers]
    lat_rows = []
    if plat and len(au) == 1:
        a = ids.index(au[0])
        lat_rows = list(range(a + 1, a + 1 + n_prompt_latents))
    return ids, {"spk": spk_rows, "latent": lat_rows}
