"""S2-Pro dual-AR weights: slow AR (text model) + fast AR (audio decoder).

* ``slow``: DecoderLM (dense, tied embeddings, pairwise RoPE, QK-norm).
* ``fast``: DecoderLM over codebook tokens; ``fast.embed`` is the audio
  decoder's ``embeddings`` table (shared by all codebooks) and ``fast.lm_head``
  its ``output`` head.
* ``codebook_embeddings`` [num_codebooks * codebook_size, text_dim]: the VQ
  embedding added to the slow AR's input at VQ positions.
* ``sem_head`` [codebook_size + 1, text_dim]: the rows of the tied LM head
  that constrained decoding can pick (the contiguous semantic tokens, then
  <|im_end|>).  The reference computes all 155776 logits and adds a -inf bias
  outside those ids (sglang_omni/models/fishaudio_s2_pro/sglang_model.py:268-274,
  353-354); sampling over the gathered rows is the same distribution at
  1/38 of the LM-head bytes.

Checkpoint names are the fish ones (``text_model.model.*``, ``audio_decoder.*``;
reference loader: sglang_model.py:386-460, modeling.py:919-1010).
"""
from __future__ import annotations

import torch
from torch import nn

from ..decoder import DecoderLM
from .hf_config import S2ProConfig


def load_fish_decoder(m: DecoderLM, sd: dict[str, torch.Tensor], prefix: str, embed_key: str,
                      head_key: str | None = None) -> None:
    """Fills a DecoderLM from fish-named tensors (``layers.N.attention.wqkv.weight`` ...)."""
    cfg = m.cfg
    cp = lambda dst, src: dst.copy_(src.to(dst.dtype))  # noqa: E731
    g = lambda k: sd[prefix + k]  # noqa: E731
    cp(m.embed, g(embed_key))
    for i, L in enumerate(m.layers):
        p = f"layers.{i}."
        cp(L.ln1, g(p + "attention_norm.weight"))
        cp(L.ln2, g(p + "ffn_norm.weight"))
        cp(L.qkv, g(p + "attention.wqkv.weight"))
        cp(L.o, g(p + "attention.wo.weight"))
        if cfg.qk_norm:
            cp(L.q_norm, g(p + "attention.q_norm.weight"))
            cp(L.k_norm, g(p + "attention.k_norm.weight"))
        cp(L.mlp13, torch.cat([g(p + "feed_forward.w1.weight"), g(p + "feed_forward.w3.weight")], 0))
        cp(L.mlp2, g(p + "feed_forward.w2.weight"))
    cp(m.final_norm, g("norm.weight"))
    if m.lm_head is not None and head_key is not None:
        cp(m.lm_head, g(head_key))


class S2ProDualAR(nn.Module):
    def __init__(self, cfg: S2ProConfig, device="cpu"):
        super().__init__()
        self.cfg = cfg
        sc, fc = cfg.slow, cfg.fast
        self.slow = DecoderLM(sc, device)
        self.fast = DecoderLM(fc, device)
        dt = sc.dtype
        P = lambda *s: nn.Parameter(torch.empty(*s, dtype=dt, device=device), requires_grad=False)  # noqa: E731
        self.has_project_in = fc.hidden_size != sc.hidden_size
        if self.has_project_in:
            self.project_in_w = P(fc.hidden_size, sc.hidden_size)
            self.project_in_b = P(fc.hidden_size)
        self.codebook_embeddings = P(cfg.num_codebooks * cfg.codebook_size, sc.hidden_size)
        self.register_buffer("sem_head", torch.empty(cfg.codebook_size + 1, sc.hidden_size, dtype=dt, device=device),
                             persistent=False)

    @torch.no_grad()
    def refresh_semantic_head(self):
        c = self.cfg
        w = self.slow.head_weight
        self.sem_head[: c.codebook_size].copy_(w[c.semantic_begin_id: c.semantic_begin_id + c.codebook_size])
        self.sem_head[c.codebook_size].copy_(w[c.im_end_id])

    @torch.no_grad()
    def random_init_(self, seed: int = 0, std: float = 0.02):
        self.slow.random_init_(seed=seed, std=std)
        self.fast.random_init_(seed=seed + 1, std=std)
        dev = self.codebook_embeddings.device
        g = torch.Generator(device=dev).manual_seed(seed * 7 + 3)
        self.codebook_embeddings.normal_(0.0, std, generator=g)
        if self.has_project_in:
            self.project_in_w.normal_(0.0, std, generator=g)
            self.project_in_b.zero_()
        self.refresh_semantic_head()
        return self

    @torch.no_grad()
    def load_state_dict_fish(self, sd: dict[str, torch.Tensor]):
        load_fish_decoder(self.slow, sd, "text_model.model.", "embeddings.weight",
                          None if self.cfg.slow.tie_word_embeddings else "output.weight")
        ad = "audio_decoder."
        load_fish_decoder(self.fast, sd, ad, "embeddings.weight", "output.weight")
        self.codebook_embeddings.copy_(sd[ad + "codebook_embeddings.weight"].to(self.codebook_embeddings.dtype))
        if self.has_project_in:
            self.project_in_w.copy_(sd[ad + "project_in.weight"].to(self.project_in_w.dtype))
            self.project_in_b.copy_(sd[ad + "project_in.bias"].to(self.project_in_b.dtype))
        self.refresh_semantic_head()
