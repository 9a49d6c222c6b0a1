"""Host-side fault injection for the control plane (tests of failure handling).

``inject(rules)`` wraps every PUSH socket the control plane creates from then
on (local queues and ZMQ alike) so that matching messages are dropped, delayed
or duplicated, or have their relay metadata corrupted.  A rule matches a
message type (``complete`` / ``stream`` / ``data_ready`` / ``submit``), optionally
the sending stage (``from_stage``) and the destination endpoint substring
(``to``); ``count`` limits how many messages it hits (-1 = all).

Nothing here touches a GPU: faults are made on the host, where the pipeline
must turn them into request errors (a lost completion runs into the
coordinator's request deadline, a corrupted relay descriptor fails the one
request at the receiving stage) or absorb them (duplicated chunks are dropped
by sequence number, delays only delay).

The reference has no injector besides SGLang's forced-retraction knob
(sglang_omni/engines/ar/sglang_backend/scheduler/decode.py:10-11,37-38).
"""
from __future__ import annotations

import asyncio
import copy
from dataclasses import dataclass, field

from ..proto import CompleteMessage, DataReadyMessage, StreamMessage, SubmitMessage

_KIND = {CompleteMessage: "complete", StreamMessage: "stream", DataReadyMessage: "data_ready",
         SubmitMessage: "submit"}


@dataclass
class FaultRule:
    action: str                  # drop | delay | duplicate | corrupt
    kind: str                    # complete | stream | data_ready | submit
    from_stage: str | None = None
    to: str | None = None
    count: int = 1               # messages to hit; -1 = every match
    delay_s: float = 0.05
    hits: int = field(default=0, compare=False)

    def matches(self, msg, endpoint: str) -> bool:
        if self.count >= 0 and self.hits >= self.count:
            return False
        if _KIND.get(type(msg)) != self.kind:
            return False
        if self.from_stage is not None and getattr(msg, "from_stage", None) != self.from_stage:
            return False
        return self.to is None or self.to in endpoint


_RULES: list[FaultRule] = []


def inject(rules: list[FaultRule]) -> None:
    """Installs rules for sockets created from now on (process-wide)."""
    _RULES.extend(rules)


def clear() -> None:
    _RULES.clear()


def active() -> bool:
    return bool(_RULES)


def _corrupt_value(v):
    if isinstance(v, dict):
        return {k: _corrupt_value(x) for k, x in v.items()}
    if isinstance(v, (list, tuple)):
        return type(v)(_corrupt_value(x) for x in v)
    if isinstance(v, bool):
        return v
    if isinstance(v, int):
        return v + (1 << 40)                 # offsets / sizes far outside any segment
    if isinstance(v, str):
        return v + "-corrupt"                # segment names that do not exist
    if isinstance(v, (bytes, bytearray)):
        return bytes(v[: len(v) // 2])       # a truncated inline payload
    return v


def _corrupt(msg):
    bad = copy.copy(msg)
    md = bad.shm_metadata
    bad.shm_metadata = _corrupt_value(md) if md is not None else {"corrupt": True}
    return bad


class FaultyPush:
    """Wraps a PUSH socket: applies the matching rule to each outgoing message."""

    def __init__(self, inner, endpoint: str):
        self.inner = inner
        self.endpoint = endpoint

    async def send(self, msg) -> None:
        for rule in _RULES:
            if rule.matches(msg, self.endpoint):
                rule.hits += 1
                if rule.action == "drop":
                    return
                if rule.action == "delay":
                    await asyncio.sleep(rule.delay_s)
                    break
                if rule.action == "duplicate":
                    await self.inner.send(msg)
                    break
                if rule.action == "corrupt" and isinstance(msg, DataReadyMessage):
                    msg = _corrupt(msg)
                    break
        await self.inner.send(msg)

    def close(self):
        self.inner.close()
