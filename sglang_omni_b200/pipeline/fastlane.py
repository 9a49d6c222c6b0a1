"""In-process fast lanes between streaming stages.

A stage's per-token stream to the next stage normally travels as control
messages through the event loop (relay write, DataReady message, the receiving
stage's mailbox, one coroutine wake-up per item).  When producer and consumer
run in the same process (the single-process pipeline runner), the consumer
registers a *lane* under its stage name and the producer's engine thread hands
items to it directly (``deliver_many``), without touching the event loop.
The thinker -> talker token stream and the talker -> code2wav frame stream of
the speech pipeline use it: per step they carry one item per active stream,
which at 32 streams was most of the event loop's work and sat on the
time-to-first-audio path.  Start / end-of-stream signals and errors still go
through the regular stage channels (they are rare and ordered after the data).

Stages in other processes are not registered here, so their producers fall
back to the relay path.
"""
from __future__ import annotations

import threading

_lock = threading.Lock()
_lanes: dict[str, object] = {}


def register(stage: str, lane) -> None:
    """``lane.deliver_many(items)``: items = [(request_id, data dict), ...], thread-safe."""
    with _lock:
        _lanes[stage] = lane


def unregister(stage: str, lane) -> None:
    with _lock:
        if _lanes.get(stage) is lane:
            del _lanes[stage]


def get(stage: str | None):
    if stage is None:
        return None
    with _lock:
        return _lanes.get(stage)
