"""Paged GQA attention (csrc/attention.cu) and the KV-cache layout helpers.

KV cache of one layer: ``[pages, Hkv, 64, D]`` bf16 (page size 64); a request
owns a row of page ids in ``block_table``; token slot = page * 64 + offset.

Reference counterparts: SGLang RadixAttention backends (FlashInfer / FA3) as
used by sglang_omni/models/qwen3_omni/thinker.py:236-243, and the encoders'
non-causal SDPA (transformers qwen3_omni_moe audio / vision towers).
"""
from __future__ import annotations

import math
import os
import threading
from collections import OrderedDict

import torch
import torch.nn.functional as F

from . import _check
from ._ext import ext, status_word

PAGE = 64


def prefill_tile_rows(head_dim: int, group: int, paged: bool = True, window: int = 0) -> int:
    """Packed query rows per tile of the prefill kernel that serves this shape: 256 (or 128 with
    OMNI_FA_TILE_ROWS=128) for the tcgen05 kernels (paged K/V, head_dim 128, no sliding
    window, G | 128), else 64 for the mma.sync kernel.  OMNI_FA_SM100=0 keeps the 64-row
    kernel everywhere."""
    if os.environ.get("OMNI_FA_SM100", "1") == "0":
        return 64
    if not (paged and head_dim == 128 and window == 0 and 128 % max(1, group) == 0):
        return 64
    # 256: two 128-row tiles per CTA whose softmax and tensor-core work overlap; 128: one tile
    return int(os.environ.get("OMNI_FA_TILE_ROWS", "256"))


def prefill_tiles(q_lens: list[int], group: int, rows: int = 64) -> tuple[list[int], list[int]]:
    """Query tiles of the GQA-packed prefill kernels: (request, first token) per tile of
    `rows` packed rows (rows / group tokens)."""
    tpt = max(1, rows // group)
    req, tok0 = [], []
    for b, n in enumerate(q_lens):
        for t in range(0, n, tpt):
            req.append(b)
            tok0.append(t)
    return req, tok0


def _sdpa_ref(q, k, v, causal, q_offset, scale, window=0):
    """q [Tq, Hq, D], k/v [Tk, Hkv, D] -> [Tq, Hq, D] in fp32 (window > 0: causal sliding window)."""
    hq, hkv = q.shape[1], k.shape[1]
    g = hq // hkv
    k = k.float().repeat_interleave(g, dim=1)
    v = v.float().repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), k) * scale
    if causal:
        tq, tk = q.shape[0], k.shape[0]
        qi = torch.arange(tq, device=q.device)[:, None] + q_offset
        ki = torch.arange(tk, device=q.device)[None, :]
        s = s.masked_fill((ki > qi)[None], float("-inf"))
        if window > 0:
            s = s.masked_fill((ki <= qi - window)[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,khd->qhd", p, v)


def gather_kv_ref(cache: torch.Tensor, pages: list[int] | torch.Tensor, n: int) -> torch.Tensor:
    """[n, Hkv, D] keys (or values) of one request from a paged cache [pages, Hkv, 64, D]."""
    pages = torch.as_tensor(pages, dtype=torch.long, device=cache.device)
    need = (n + PAGE - 1) // PAGE
    blk = cache[pages[:need]]  # [need, Hkv, 64, D]
    return blk.permute(0, 2, 1, 3).reshape(need * PAGE, cache.shape[1], cache.shape[3])[:n]


def paged_attention_ref(q, k_cache, v_cache, block_table, cu_q, kv_lens, scale, causal=True, window=0):
    cu = cu_q.tolist()
    kl = kv_lens.tolist()
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    for b in range(len(kl)):
        a, e = cu[b], cu[b + 1]
        if e <= a:
            continue
        k = gather_kv_ref(k_cache, block_table[b], kl[b])
        v = gather_kv_ref(v_cache, block_table[b], kl[b])
        out[a:e] = _sdpa_ref(q[a:e], k, v, causal, kl[b] - (e - a), scale, window)
    return out


def varlen_attention_ref(q, k, v, cu_seqlens, scale, causal=False, window=0):
    cu = cu_seqlens.tolist()
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    for b in range(len(cu) - 1):
        a, e = cu[b], cu[b + 1]
        if e > a:
            out[a:e] = _sdpa_ref(q[a:e], k[a:e], v[a:e], causal, 0, scale, window)
    return out


def prefill_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                      cu_q: torch.Tensor, kv_lens: torch.Tensor, tile_req: torch.Tensor, tile_tok0: torch.Tensor,
                      num_heads: int, num_kv_heads: int, head_dim: int, scale: float | None = None,
                      out: torch.Tensor | None = None, causal: bool = True, tile_rows: int = 64,
                      window: int = 0) -> torch.Tensor:
    """Causal prefill over the paged cache. q: [T, Hq * D] rows (any row stride).

    ``tile_rows``: rows of the tiles in tile_req / tile_tok0 (``prefill_tile_rows``): 128 runs
    the tcgen05 kernel, 64 the mma.sync kernel.  ``window`` > 0 (64-row tiles only) limits
    every query to its last ``window`` keys; pages wholly below a tile's first visible key are
    never read, so a request's block-table row may reuse pages as a ring."""
    scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)
    q3 = q.view(q.shape[0], -1) if q.dim() == 2 else q
    if out is None:
        out = torch.empty(q.shape[0], num_heads * head_dim, dtype=q.dtype, device=q.device)
    if not q.is_cuda:
        ref = paged_attention_ref(q3.reshape(q.shape[0], -1)[:, : num_heads * head_dim].view(-1, num_heads, head_dim),
                                  k_cache, v_cache, block_table, cu_q, kv_lens, scale, causal, window)
        out.copy_(ref.reshape(out.shape))
        return out
    if window > 0 and tile_rows != 64:
        raise ValueError("prefill_attention: a sliding window needs the 64-row (mma.sync) tiles")
    if _check.enabled():
        _check.check_paged("attention_prefill", block_table, kv_lens, k_cache.shape[0], cu_q, q.shape[0])
        _check.check_tiles("attention_prefill", tile_req, tile_tok0, cu_q)
    ext().attention_prefill(q3, k_cache, v_cache, out, block_table, cu_q, kv_lens, None, tile_req, tile_tok0,
                            num_heads, num_kv_heads, head_dim, scale, causal, window, tile_rows, status_word(q.device))
    return out


def varlen_tile_rows(q: torch.Tensor, k: torch.Tensor, head_dim: int, group: int, window: int = 0,
                     v: torch.Tensor | None = None, out: torch.Tensor | None = None) -> int:
    """Query rows per tile for ragged attention: the tcgen05 kernels (256 or 128 rows) for head
    dims 80..128 without a sliding window and 16-byte aligned rows, else the 64-row mma.sync
    kernel (head dim 64 stays there: the tensor-core kernels would pad it to 128)."""
    if os.environ.get("OMNI_FA_SM100", "1") == "0" or window > 0 or not (80 <= head_dim <= 128) or head_dim % 16:
        return 64
    if 128 % max(1, group) or (q.stride(0) * 2) % 16 or (k.stride(0) * 2) % 16 or q.data_ptr() % 16 or \
            k.data_ptr() % 16:
        return 64
    if v is not None and (v.stride(0) != k.stride(0) or v.data_ptr() % 16):
        return 64
    if out is not None and (out.stride(0) % 8 or out.data_ptr() % 16):
        return 64
    return int(os.environ.get("OMNI_FA_TILE_ROWS", "256"))


def varlen_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor,
                     num_heads: int, num_kv_heads: int, head_dim: int, scale: float | None = None,
                     causal: bool = False, out: torch.Tensor | None = None, q_lens: list[int] | None = None,
                     tiles: tuple[torch.Tensor, torch.Tensor] | None = None, window: int = 0) -> torch.Tensor:
    """Ragged (block-diagonal) attention over contiguous q/k/v rows (encoders, vocoder transformers).

    ``window`` > 0 (with causal) limits every query to its last ``window`` keys.  ``tiles``: a
    precomputed 64-row tile table (the mma.sync kernel); without it the tile size is chosen by
    ``varlen_tile_rows`` and the table is built once per layout."""
    scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)
    T = q.shape[0]
    if out is None:
        out = torch.empty(T, num_heads * head_dim, dtype=q.dtype, device=q.device)
    if not q.is_cuda:
        ref = varlen_attention_ref(q.reshape(T, num_heads, head_dim), k.reshape(T, num_kv_heads, head_dim),
                                   v.reshape(T, num_kv_heads, head_dim), cu_seqlens, scale, causal, window)
        out.copy_(ref.reshape(out.shape))
        return out
    lens = None
    rows = 64
    if tiles is None:
        if q_lens is None:
            cu = cu_seqlens.tolist()
            q_lens = [cu[i + 1] - cu[i] for i in range(len(cu) - 1)]
        rows = varlen_tile_rows(q, k, head_dim, num_heads // num_kv_heads, window, v, out)
        tiles_req, tiles_tok0, lens = varlen_plan(q_lens, num_heads // num_kv_heads, q.device, rows)
        tiles = (tiles_req, tiles_tok0)
    if lens is None:
        lens = (cu_seqlens[1:] - cu_seqlens[:-1]).to(torch.int32)
    if _check.enabled():
        _check.check_range("varlen_attention", "cu_seqlens", cu_seqlens, 0, T + 1)
        if bool((lens < 0).any()):
            raise _check.LaunchCheckError("varlen_attention: cu_seqlens not monotone")
        _check.check_tiles("varlen_attention", tiles[0], tiles[1], cu_seqlens)
    ext().attention_prefill(q, k, v, out, None, cu_seqlens, lens, cu_seqlens, tiles[0], tiles[1],
                            num_heads, num_kv_heads, head_dim, scale, causal, window, rows, status_word(q.device))
    return out


_PLANS: "OrderedDict[tuple, tuple]" = OrderedDict()
_PLANS_LOCK = threading.Lock()
_PLANS_MAX = 64


def varlen_plan(q_lens: list[int], group: int, device, rows: int = 64) -> tuple[torch.Tensor, torch.Tensor,
                                                                                torch.Tensor]:
    """Device tile table (request, first token) and lengths of a ragged batch, built once per
    (lengths, group, device) and reused: an encoder calls the attention once per layer with the
    same layout, and a fresh host-to-device upload per layer would stall the host on the stream."""
    device = torch.device(device)
    key = (tuple(int(n) for n in q_lens), int(group), device.index, int(rows))
    with _PLANS_LOCK:
        hit = _PLANS.get(key)
        if hit is not None:
            _PLANS.move_to_end(key)
            return hit[:3]
    req, tok0 = prefill_tiles(list(key[0]), group, rows)
    n = len(req)
    host = torch.tensor(req + tok0 + list(key[0]), dtype=torch.int32)
    if device.type == "cuda":
        host = host.pin_memory()
    dev = host.to(device, non_blocking=True)
    plan = (dev[:n], dev[n:2 * n], dev[2 * n:], host)   # the pinned source lives as long as the plan
    with _PLANS_LOCK:
        _PLANS[key] = plan
        while len(_PLANS) > _PLANS_MAX:
            _PLANS.popitem(last=False)
    return plan[:3]


_SM_COUNT: dict = {}


def _resident_decode_ctas(device, head_dim: int) -> int:
    """CTAs of the decode kernel that fit on the GPU at once (shared memory bound)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SM_COUNT:
        _SM_COUNT[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SM_COUNT[idx] * (3 if head_dim > 64 else 6)


# Keys per split of decode batches whose (request, KV head) pairs alone fill the GPU.
FILL_SPLIT_KEYS = 2048


class DecodeWorkspace:
    """Split-KV scratch of the decode kernel, sized for a max batch / context."""

    def __init__(self, max_batch: int, num_heads: int, head_dim: int, max_context: int, device,
                 keys_per_split: int = 256):
        self.keys_per_split = keys_per_split
        self.max_context = max_context
        self.max_splits = max(1, (max_context + keys_per_split - 1) // keys_per_split)
        self.part_o = torch.empty(max_batch * num_heads * self.max_splits * head_dim, dtype=torch.float32,
                                  device=device)
        self.part_lse = torch.empty(max_batch * num_heads * self.max_splits, dtype=torch.float32, device=device)
        # split arrival counters: the last split of a (request, KV head) merges in the same launch
        self.counters = torch.zeros(max_batch * num_heads, dtype=torch.int32, device=device)


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                     kv_lens: torch.Tensor, num_heads: int, num_kv_heads: int, head_dim: int,
                     workspace: DecodeWorkspace | None = None, scale: float | None = None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """One query token per request. q: [B, >= Hq * D] rows."""
    scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)
    B = kv_lens.shape[0]
    if out is None:
        out = torch.empty(B, num_heads * head_dim, dtype=q.dtype, device=q.device)
    if not q.is_cuda:
        cu = torch.arange(B + 1, dtype=torch.int32)
        ref = paged_attention_ref(q.reshape(B, -1)[:, : num_heads * head_dim].view(B, num_heads, head_dim),
                                  k_cache, v_cache, block_table, cu, kv_lens, scale, True)
        out.copy_(ref.reshape(out.shape))
        return out
    if workspace is None:
        max_ctx = int(kv_lens.max().item())
        workspace = DecodeWorkspace(B, num_heads, head_dim, max_ctx, q.device)
    if _check.enabled():
        _check.check_paged("attention_decode", block_table, kv_lens, k_cache.shape[0])
    # Batches of 128 or more pairs that do not take the single split below still fill most of the
    # GPU: twice the keys per split halves the per-split setup and merge work.  The split count
    # stays within the workspace's max_splits, which was sized for the finer split.
    # When the (request, KV head) pairs alone fill more than half of the resident CTA slots
    # (148 SMs x 3 CTAs of 68 KB at head_dim 128, 6 at 64), any split adds a partial wave and
    # the merge: one split per pair is fastest (64 x 4 pairs at 1.1-1.3 k context: 41-46 us vs
    # 52-56 us at 512 keys per split, 56-62 us at 256).
    # The rule looks only at shapes known when a decode graph is captured, not at the context
    # lengths of one step: GPU-filling batches take splits of FILL_SPLIT_KEYS keys, so contexts up
    # to that length run as one split per pair while one much longer context (a skewed batch)
    # still spreads over several CTAs instead of one CTA walking all of it.  The splits past a
    # request's length exit at once.
    kps, splits = workspace.keys_per_split, workspace.max_splits
    if 2 * B * num_kv_heads > _resident_decode_ctas(q.device, head_dim):
        kps = max(kps, FILL_SPLIT_KEYS)
    elif B * num_kv_heads >= 128 and kps < 512:
        kps = 2 * kps
    # no grid slots for splits that no context within the workspace's bound can use
    splits = max(1, min(splits, -(-getattr(workspace, "max_context", kps * splits) // kps)))
    ext().attention_decode(q, k_cache, v_cache, out, block_table, kv_lens, num_heads, num_kv_heads, head_dim, scale,
                           kps, splits, workspace.part_o, workspace.part_lse,
                           getattr(workspace, "counters", None))
    return out
