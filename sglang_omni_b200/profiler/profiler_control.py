"""Broadcasts profiler start / stop to every stage through the coordinator
(sglang_omni/profiler/profiler_control.py:15-75)."""
from __future__ import annotations

import os
import time


class ProfilerControlClient:
    def __init__(self, coordinator, root: str | None = None):
        self.coordinator = coordinator
        self.root = root or os.environ.get("SGLANG_TORCH_PROFILER_DIR", "/tmp/sglang_omni_b200_profiles")

    async def start(self, run_id: str | None = None) -> str:
        run_id = run_id or time.strftime("%Y%m%d-%H%M%S")
        await self.coordinator.start_profile(run_id, os.path.join(self.root, "{run_id}", "{stage}", "trace"))
        return run_id

    async def stop(self, run_id: str) -> None:
        await self.coordinator.stop_profile(run_id)
