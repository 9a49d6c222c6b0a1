from .base import AsyncModuleEngine

__all__ = ["AsyncModuleEngine"]
