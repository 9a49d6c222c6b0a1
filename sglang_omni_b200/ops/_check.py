"""Host-side validation of the index inputs of every kernel launch.

Enabled with ``OMNI_DEVICE_CHECKS=1``.  Each check copies the small index
tensors of one launch (block tables, slot mappings, token ids, offsets) to the
host and raises ``LaunchCheckError`` naming the op and the first bad entry
*before* the kernel runs, so an out-of-range index is reported as a Python
exception instead of reaching the GPU.  Checks are skipped while a CUDA graph
is being captured (a capture cannot synchronise); run with
``OMNI_USE_CUDA_GRAPHS=0`` to check every step.  Every check synchronises, so
this mode is for debugging only.
"""
from __future__ import annotations

import torch

from ..environ import environ

_on: bool | None = None


class LaunchCheckError(RuntimeError):
    pass


def enabled() -> bool:
    global _on
    if _on is None:
        _on = bool(environ.OMNI_DEVICE_CHECKS.get())
    if not _on:
        return False
    return not torch.cuda.is_current_stream_capturing()


def set_enabled(flag: bool) -> None:
    global _on
    _on = flag


def _fail(op: str, msg: str):
    raise LaunchCheckError(f"{op}: {msg}")


def _h(t: torch.Tensor):
    return t.detach().to("cpu", torch.int64)


def check_paged(op: str, block_table: torch.Tensor, kv_lens: torch.Tensor, num_pages: int,
                cu_q: torch.Tensor | None = None, q_rows: int | None = None):
    bt, kl = _h(block_table), _h(kv_lens)
    if bt.dim() != 2 or bt.shape[0] < kl.shape[0]:
        _fail(op, f"block table {tuple(bt.shape)} for {kl.shape[0]} requests")
    for b in range(kl.shape[0]):
        n = int(kl[b])
        if n < 0:
            _fail(op, f"request {b}: kv_len {n} < 0")
        need = (n + 63) // 64
        if need > bt.shape[1]:
            _fail(op, f"request {b}: kv_len {n} needs {need} pages, block table has {bt.shape[1]}")
        if need:
            row = bt[b, :need]
            bad = (row < 0) | (row >= num_pages)
            if bool(bad.any()):
                i = int(bad.nonzero()[0])
                _fail(op, f"request {b}: block_table[{i}] = {int(row[i])} outside [0, {num_pages})")
    if cu_q is not None:
        cu = _h(cu_q)
        if int(cu[0]) != 0 or bool((cu[1:] < cu[:-1]).any()):
            _fail(op, f"cu_q not monotone from 0: {cu.tolist()[:8]}")
        if q_rows is not None and int(cu[-1]) > q_rows:
            _fail(op, f"cu_q ends at {int(cu[-1])} > {q_rows} query rows")
        ql = cu[1:] - cu[:-1]
        if bool((ql > kl[: ql.shape[0]]).any()):
            b = int((ql > kl[: ql.shape[0]]).nonzero()[0])
            _fail(op, f"request {b}: {int(ql[b])} queries but kv_len {int(kl[b])}")


def check_tiles(op: str, tile_req: torch.Tensor, tile_tok0: torch.Tensor, cu_q: torch.Tensor):
    tr, tt, cu = _h(tile_req), _h(tile_tok0), _h(cu_q)
    B = cu.shape[0] - 1
    if tr.shape != tt.shape:
        _fail(op, "tile arrays differ in length")
    if tr.numel() and (int(tr.min()) < 0 or int(tr.max()) >= B):
        _fail(op, f"tile_req outside [0, {B})")
    for i in range(tr.numel()):
        b = int(tr[i])
        if int(tt[i]) < 0 or int(tt[i]) >= int(cu[b + 1] - cu[b]):
            _fail(op, f"tile {i}: first token {int(tt[i])} outside request {b} of {int(cu[b + 1] - cu[b])} rows")


def check_range(op: str, name: str, t: torch.Tensor, lo: int, hi: int, allow: int | None = None):
    v = _h(t).reshape(-1)
    if v.numel() == 0:
        return
    bad = (v < lo) | (v >= hi)
    if allow is not None:
        bad &= v != allow
    if bool(bad.any()):
        i = int(bad.nonzero()[0])
        _fail(op, f"{name}[{i}] = {int(v[i])} outside [{lo}, {hi})")


def check_offsets(op: str, offsets: torch.Tensor, rows: int):
    o = _h(offsets)
    # a sub-range of experts (tensor-parallel MoE) starts past row 0
    if int(o[0]) < 0 or bool((o[1:] < o[:-1]).any()) or int(o[-1]) > rows:
        _fail(op, f"group offsets not monotone within [0, {rows}]: first {o.tolist()[:6]} last {int(o[-1])}")
