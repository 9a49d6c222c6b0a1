"""Per-stage torch.profiler session (CPU + CUDA, shapes, memory, stack, flops)
with one long active window; the Chrome trace is written on stop and gzipped
in the background.  Start / stop arrive as control messages
(sglang_omni/profiler/torch_profiler.py:24-179).  Unlike the reference, a
second start while active is a no-op instead of an error."""
from __future__ import annotations

import gzip
import os
import shutil
import threading

import torch


class ProfilerBase:
    def start(self) -> None: ...

    def stop(self) -> str | None: ...


class TorchProfiler(ProfilerBase):
    def __init__(self, trace_path: str):
        self.trace_path = trace_path
        self._prof = None

    def start(self):
        if self._prof is not None:
            return
        acts = [torch.profiler.ProfilerActivity.CPU]
        if torch.cuda.is_available():
            acts.append(torch.profiler.ProfilerActivity.CUDA)
        self._prof = torch.profiler.profile(activities=acts, record_shapes=True, profile_memory=True,
                                            with_stack=True, with_flops=True)
        self._prof.__enter__()

    def stop(self) -> str | None:
        if self._prof is None:
            return None
        prof, self._prof = self._prof, None
        prof.__exit__(None, None, None)
        os.makedirs(os.path.dirname(self.trace_path) or ".", exist_ok=True)
        path = self.trace_path + ".json"
        prof.export_chrome_trace(path)

        def _gz():
            with open(path, "rb") as f, gzip.open(path + ".gz", "wb") as g:
                shutil.copyfileobj(f, g)
            os.remove(path)

        threading.Thread(target=_gz, daemon=True).start()
        return path + ".gz"
