"""Architecture name -> PipelineConfig class registry.

Every ``sglang_omni_b200.models.<pkg>.config`` module that defines
``EntryClass`` (a PipelineConfig subclass with a class-level ``architecture``
and optional ``Variants``) is discovered on first use, like
sglang_omni/models/registry.py:14-90.
"""
from __future__ import annotations

import importlib
import logging
import pkgutil

log = logging.getLogger(__name__)


class PipelineConfigRegistry:
    def __init__(self):
        self._by_arch: dict[str, type] = {}
        self._loaded = False

    def _load(self):
        if self._loaded:
            return
        self._loaded = True
        from .. import models as pkg

        for m in pkgutil.iter_modules(pkg.__path__):
            if not m.ispkg:
                continue
            try:
                mod = importlib.import_module(f"{pkg.__name__}.{m.name}.config")
            except ModuleNotFoundError:
                continue
            except Exception:
                log.exception("failed to import %s.config", m.name)
                continue
            entries = getattr(mod, "EntryClass", None)
            if entries is None:
                continue
            for cls in entries if isinstance(entries, (list, tuple)) else [entries]:
                self.register(cls)

    def register(self, cls):
        archs = getattr(cls, "architectures", None) or [getattr(cls, "architecture", None)]
        for a in archs:
            if a:
                self._by_arch[a] = cls
        return cls

    def get_config(self, architecture: str, variant: str | None = None):
        self._load()
        cls = self._by_arch.get(architecture)
        if cls is None:
            raise KeyError(f"no pipeline registered for architecture {architecture!r}; "
                           f"known: {sorted(self._by_arch)}")
        variants = getattr(cls, "Variants", None)
        if variant and variants:
            if variant not in variants:
                raise KeyError(f"{cls.__name__} has no variant {variant!r}; known: {sorted(variants)}")
            cls = variants[variant]
        return cls

    def architectures(self) -> list[str]:
        self._load()
        return sorted(self._by_arch)


PIPELINE_CONFIG_REGISTRY = PipelineConfigRegistry()
