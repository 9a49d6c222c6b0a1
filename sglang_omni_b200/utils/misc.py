"""Small shared helpers (import_string, seeding, layer ids, pickled broadcast).

Reference counterparts: sglang_omni/utils/misc.py:17-102.
"""
from __future__ import annotations

import importlib
import io
import pickle
import random
import re
from typing import Any

import numpy as np
import torch

_REF_PREFIX = "sglang_omni."
_OWN_PREFIX = "sglang_omni_b200."


def import_string(path: str) -> Any:
    """Imports ``pkg.module.attr``.  Paths written for the reference package
    (``sglang_omni.*``) resolve to the same-named object of this package."""
    if path.startswith(_REF_PREFIX) and not path.startswith(_OWN_PREFIX):
        try:
            return import_string(_OWN_PREFIX + path[len(_REF_PREFIX):])
        except (ImportError, AttributeError):
            pass
    mod, _, attr = path.rpartition(".")
    if not mod:
        raise ImportError(f"not a dotted path: {path!r}")
    m = importlib.import_module(mod)
    try:
        return getattr(m, attr)
    except AttributeError as exc:
        raise ImportError(f"{mod} has no attribute {attr!r}") from exc


def get_layer_id(name: str) -> int | None:
    m = re.search(r"layers\.(\d+)\.", name)
    return int(m.group(1)) if m else None


def set_random_seed(seed: int) -> None:
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


def broadcast_pyobj(obj: Any, rank: int, src: int = 0, group=None, device="cpu") -> Any:
    """Pickles `obj` on `src` and broadcasts it with torch.distributed."""
    import torch.distributed as dist

    if rank == src:
        buf = io.BytesIO()
        pickle.dump(obj, buf)
        data = torch.frombuffer(bytearray(buf.getvalue()), dtype=torch.uint8).to(device)
        size = torch.tensor([data.numel()], dtype=torch.long, device=device)
        dist.broadcast(size, src, group=group)
        dist.broadcast(data, src, group=group)
        return obj
    size = torch.tensor([0], dtype=torch.long, device=device)
    dist.broadcast(size, src, group=group)
    data = torch.empty(int(size.item()), dtype=torch.uint8, device=device)
    dist.broadcast(data, src, group=group)
    return pickle.loads(data.cpu().numpy().tobytes())
