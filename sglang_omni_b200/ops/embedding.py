"""Token-embedding gather with multimodal row overwrite (csrc/fused_ops.cu).

Reference counterpart: SGLangModelRunner._inject_multimodal_embeds,
sglang_omni/engines/omni/runtime/sglang_ar.py:548-701 (scatter of encoder
embeddings into the image / audio / video placeholder positions).
"""
from __future__ import annotations

import torch

from . import _check
from ._ext import ext


def embed(ids: torch.Tensor, table: torch.Tensor, mm_index: torch.Tensor | None = None,
          mm_embeds: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    if not ids.is_cuda:
        y = table[ids.long()].clone()
        if mm_index is not None:
            sel = mm_index >= 0
            if bool(sel.any()):
                y[sel] = mm_embeds[mm_index[sel].long()].to(y.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=ids.device)
    if _check.enabled():
        if mm_index is not None:
            _check.check_range("embed", "mm_index", mm_index, 0, mm_embeds.shape[0], allow=-1)
            _check.check_range("embed", "ids", ids[mm_index < 0], 0, table.shape[0])
        else:
            _check.check_range("embed", "ids", ids, 0, table.shape[0])
    ext().embed(ids, table, out, mm_index, mm_embeds)
    return out


def vq_embed_ref(table, codebooks, codes, cb_size, scale, sem_lo, sem_hi, ids=None, slot=None, slot_tokens=None,
                 code_row=None):
    """PyTorch restatement of :func:`vq_embed` (the kernel's oracle)."""
    if slot is not None:
        sl = slot.long()
        tok = slot_tokens[sl].long()
        rows = sl if code_row is None else code_row.long()
    else:
        tok = ids.long()
        rows = torch.arange(tok.numel(), device=tok.device) if code_row is None else code_row.long()
    e = table[tok]
    if code_row is not None:
        vq = rows >= 0
    else:
        vq = (tok >= sem_lo) & (tok <= sem_hi)
    out = e.clone()
    if bool(vq.any()):
        r = rows[vq]
        c = codes[r].long().clamp(0, cb_size - 1)
        ncb = c.shape[1]
        off = torch.arange(ncb, device=c.device) * cb_size
        s = codebooks[c + off].float().sum(1).to(e.dtype)
        out[vq] = ((e[vq] + s) * scale).to(e.dtype)
    return out


def vq_embed(table: torch.Tensor, codebooks: torch.Tensor, codes: torch.Tensor, cb_size: int, scale: float,
             sem_lo: int, sem_hi: int, ids: torch.Tensor | None = None, slot: torch.Tensor | None = None,
             slot_tokens: torch.Tensor | None = None, code_row: torch.Tensor | None = None,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """Dual-AR input rows: E[id], and at VQ positions (E[id] + sum_c CB[c*cb_size + code_c]) * scale.

    Prefill passes ``ids`` and ``code_row`` (row of ``codes`` per token, -1 for
    text); decode passes ``slot`` + ``slot_tokens`` (the previous token of each
    slot) and per-slot ``codes``, and VQ positions are the ids in [sem_lo, sem_hi].
    Reference: FishQwen3AudioDecoder.embed_text_dim / embed_one_token
    (sglang_omni/models/fishaudio_s2_pro/fish_speech/models/text2semantic/modeling.py:1040-1110)
    and the decode-time combination in sglang_model.py:306-317.
    """
    n = (ids if ids is not None else slot).numel()
    if out is None:
        out = torch.empty(n, table.shape[1], dtype=table.dtype, device=table.device)
    if not table.is_cuda:
        out.copy_(vq_embed_ref(table, codebooks, codes, cb_size, scale, sem_lo, sem_hi, ids, slot, slot_tokens,
                               code_row))
        return out
    if _check.enabled():
        if ids is not None:
            _check.check_range("vq_embed", "ids", ids, 0, table.shape[0])
        else:
            _check.check_range("vq_embed", "slot", slot, 0, slot_tokens.shape[0])
            _check.check_range("vq_embed", "slot_tokens", slot_tokens[slot.long()], 0, table.shape[0])
        if code_row is not None:
            _check.check_range("vq_embed", "code_row", code_row, 0, codes.shape[0], allow=-1)
    ext().vq_embed(ids, slot, slot_tokens, table, codebooks, codes, code_row, sem_lo, sem_hi, cb_size, scale, out)
    return out
