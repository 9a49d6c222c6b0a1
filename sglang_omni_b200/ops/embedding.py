"""Token-embedding gather with multimodal row overwrite (csrc/fused_ops.cu).

Reference counterpart: SGLangModelRunner._inject_multimodal_embeds,
sglang_omni/engines/omni/runtime/sglang_ar.py:548-701 (scatter of encoder
embeddings into the image / audio / video placeholder positions).
"""
from __future__ import annotations

import torch

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
    ext().embed(ids, table, out, mm_index, mm_embeds)
    return out
