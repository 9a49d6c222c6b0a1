"""ConfigManager: resolve a PipelineConfig from a model path (HF
``architectures[0]`` -> registry) or a YAML file, and apply dotted CLI
overrides (``--stages.4.executor.args.max_batch 32``).

Reference: sglang_omni/config/manager.py:11-125.  Type inference here also
parses floats (the reference's ``isnumeric`` check never matches them).
"""
from __future__ import annotations

import json
import os
from typing import Any

import yaml

from ..models.registry import PIPELINE_CONFIG_REGISTRY
from ..utils.misc import import_string
from .schema import PipelineConfig


def _convert(v: str) -> Any:
    low = v.lower()
    if low in ("true", "false"):
        return low == "true"
    if low in ("none", "null"):
        return None
    try:
        return int(v)
    except ValueError:
        pass
    try:
        return float(v)
    except ValueError:
        pass
    if v.startswith(("[", "{")):
        try:
            return json.loads(v)
        except json.JSONDecodeError:
            return v
    return v


class ConfigManager:
    @staticmethod
    def parse_extra_args(args: list[str]) -> dict[str, Any]:
        out: dict[str, Any] = {}
        i = 0
        while i < len(args):
            a = args[i]
            if not a.startswith("--"):
                i += 1
                continue
            key = a[2:]
            if "=" in key:
                key, val = key.split("=", 1)
            elif i + 1 < len(args) and not args[i + 1].startswith("--"):
                val = args[i + 1]
                i += 1
            else:
                val = "true"
            out[key.replace("-", "_")] = _convert(val)
            i += 1
        return out

    @staticmethod
    def merge_config(cfg: PipelineConfig, overrides: dict[str, Any]) -> PipelineConfig:
        data = cfg.model_dump()
        for dotted, val in overrides.items():
            cur = data
            parts = dotted.split(".")
            for p in parts[:-1]:
                cur = cur[int(p)] if isinstance(cur, list) else cur.setdefault(p, {})
            last = parts[-1]
            if isinstance(cur, list):
                cur[int(last)] = val
            else:
                cur[last] = val
        return type(cfg)(**data)

    @staticmethod
    def from_model_path(model_path: str, variant: str | None = None, **kw) -> PipelineConfig:
        """``model_path``: a checkpoint directory or a Hugging Face Hub repository id (resolved to
        its local snapshot, downloaded unless offline); the config keeps the path as given."""
        from ..models.model_path import resolve_model_path

        arch = None
        cfg_file = os.path.join(resolve_model_path(model_path), "config.json")
        if os.path.exists(cfg_file):
            with open(cfg_file) as f:
                d = json.load(f)
            archs = d.get("architectures") or []
            arch = archs[0] if archs else d.get("model_type")
        if arch is None:
            raise ValueError(f"cannot determine the architecture of {model_path!r} (no config.json)")
        cls = PIPELINE_CONFIG_REGISTRY.get_config(arch, variant)
        return cls(model_path=model_path, **kw)

    @staticmethod
    def from_file(path: str) -> PipelineConfig:
        with open(path) as f:
            data = yaml.safe_load(f)
        cls_name = data.get("config_cls")
        cls = PipelineConfig
        if cls_name and cls_name != "PipelineConfig":
            cls = _find_config_cls(cls_name) or PipelineConfig
        return cls(**data)

    @staticmethod
    def to_file(cfg: PipelineConfig, path: str) -> None:
        with open(path, "w") as f:
            yaml.safe_dump(cfg.model_dump(), f, sort_keys=False)


def _find_config_cls(name: str):
    if "." in name:
        try:
            return import_string(name)
        except ImportError:
            return None
    PIPELINE_CONFIG_REGISTRY._load()
    for cls in PIPELINE_CONFIG_REGISTRY._by_arch.values():
        if cls.__name__ == name:
            return cls
        for v in (getattr(cls, "Variants", None) or {}).values():
            if v.__name__ == name:
                return v
    return None
