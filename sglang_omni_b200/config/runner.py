"""Single-process pipeline lifecycle (sglang_omni/config/runner.py:12-63):
start the coordinator and every stage, run until one of them fails
(FIRST_EXCEPTION), stop everything."""
from __future__ import annotations

import asyncio
import os
import sys
import logging

from ..pipeline.coordinator import Coordinator
from ..pipeline.stage.runtime import Stage

log = logging.getLogger(__name__)


class PipelineRunner:
    def __init__(self, coordinator: Coordinator, stages: list[Stage]):
        self.coordinator = coordinator
        self.stages = stages
        self._tasks: list[asyncio.Task] = []

    async def start(self):
        # Engine threads of GPU stages share this interpreter with the event loop
        # that routes every stage message; a short GIL switch interval keeps the
        # loop responsive while they run Python between kernel launches.
        iv = float(os.environ.get("OMNI_GIL_SWITCH_INTERVAL_S", "0.0005"))
        if 0 < iv < sys.getswitchinterval():
            sys.setswitchinterval(iv)
        await self.coordinator.start()
        for s in self.stages:
            await s.start()
        await asyncio.sleep(0.05)  # let the abort subscribers connect
        self._tasks = [self.coordinator.start_completion_loop()]
        self._tasks += [asyncio.ensure_future(s.run()) for s in self.stages]

    async def wait(self):
        done, _ = await asyncio.wait(self._tasks, return_when=asyncio.FIRST_EXCEPTION)
        for t in done:
            if t.exception() is not None:
                raise t.exception()

    async def stop(self):
        for s in self.stages:
            try:
                await s.stop()
            except Exception:
                log.exception("stopping stage %s", s.name)
        await self.coordinator.stop()
        for t in self._tasks:
            t.cancel()

    async def __aenter__(self):
        await self.start()
        return self

    async def __aexit__(self, *exc):
        await self.stop()
