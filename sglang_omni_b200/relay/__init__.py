from .base import RELAY_REGISTRY, CreditAllocator, Relay, RelayOperation, create_relay, register_relay
from . import inproc, shm  # noqa: F401  (register the always-available backends)

__all__ = ["RELAY_REGISTRY", "CreditAllocator", "Relay", "RelayOperation", "create_relay", "register_relay"]
