"""Typed environment variables (sglang_omni/environ.py:10-107)."""
from __future__ import annotations

import os
from typing import Any, Callable, Generic, TypeVar

T = TypeVar("T")


class EnvVar(Generic[T]):
    def __init__(self, name: str, default: T, parse: Callable[[str], T] = str):
        self.name = name
        self.default = default
        self.parse = parse

    def get(self) -> T:
        v = os.environ.get(self.name)
        return self.default if v is None else self.parse(v)

    def set(self, value: Any) -> None:
        os.environ[self.name] = str(value)


def _bool(v: str) -> bool:
    return v.lower() in ("1", "true", "yes", "on")


class Environ:
    SGLOMNI_LOG_LEVEL = EnvVar("SGLOMNI_LOG_LEVEL", "INFO")
    SGLANG_OMNI_STARTUP_TIMEOUT = EnvVar("SGLANG_OMNI_STARTUP_TIMEOUT", 600.0, float)
    SGLANG_TORCH_PROFILER_DIR = EnvVar("SGLANG_TORCH_PROFILER_DIR", "/tmp/sglang_omni_b200_profiles")
    OMNI_DEVICE_CHECKS = EnvVar("OMNI_DEVICE_CHECKS", False, _bool)
    OMNI_USE_CUDA_GRAPHS = EnvVar("OMNI_USE_CUDA_GRAPHS", True, _bool)


environ = Environ()
