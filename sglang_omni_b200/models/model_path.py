"""``--model-path`` values that name a Hugging Face Hub repository ("Qwen/Qwen3-Omni-30B-A3B-
Instruct") resolve to a local snapshot directory: the Hugging Face cache first, then (unless
offline: ``HF_HUB_OFFLINE=1`` or ``local_files_only``) a download.  A cached snapshot that lacks
weight shards its index lists (an interrupted download) is fetched again once.  Local paths
and the synthetic names ("random", "toy", "") pass through unchanged.  The reference resolves
model paths the same way (sglang_omni/models/weight_loader.py:37-45 and its forced refresh of a
partial snapshot, :196-208)."""
from __future__ import annotations

import json
import os
import re

_SYNTHETIC = {"", "random", "toy"}
_REPO = re.compile(r"^[A-Za-z0-9][\w.\-]*/[\w.\-]+$")


def is_repo_id(model_path: str) -> bool:
    return bool(_REPO.match(model_path or "")) and not os.path.exists(model_path)


def snapshot_complete(path: str) -> bool:
    """Whether a checkpoint directory holds the weight files it declares (or any weights)."""
    idx = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(idx):
        with open(idx) as f:
            shards = set(json.load(f).get("weight_map", {}).values())
        return all(os.path.exists(os.path.join(path, s)) for s in shards)
    names = os.listdir(path) if os.path.isdir(path) else []
    return any(n.endswith((".safetensors", ".bin", ".pt", ".pth")) for n in names) or \
        os.path.exists(os.path.join(path, "config.json"))


def _offline(local_files_only: bool | None) -> bool:
    if local_files_only is not None:
        return local_files_only
    return os.environ.get("HF_HUB_OFFLINE", "").lower() in ("1", "true", "yes")


_RESOLVED: dict[str, str] = {}


def resolve_model_path(model_path: str, local_files_only: bool | None = None) -> str:
    if not model_path or model_path in _SYNTHETIC or not is_repo_id(model_path):
        return model_path
    if model_path in _RESOLVED:
        return _RESOLVED[model_path]
    from huggingface_hub import snapshot_download

    offline = _offline(local_files_only)
    path = None
    try:
        path = snapshot_download(model_path, local_files_only=True)
    except Exception as exc:
        if offline:
            raise FileNotFoundError(f"{model_path!r} is neither a local directory nor in the Hugging Face cache "
                                    f"(offline): {exc}") from exc
    if path is None or not snapshot_complete(path):
        if offline:
            raise FileNotFoundError(f"the cached snapshot of {model_path!r} at {path} is missing weight files "
                                    f"(offline, cannot fetch them)")
        path = snapshot_download(model_path, force_download=path is not None)
    _RESOLVED[model_path] = path
    return path
