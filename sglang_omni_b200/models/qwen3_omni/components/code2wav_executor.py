"""Reference factory path of the Code2Wav stage
(sglang_omni/models/qwen3_omni/components/code2wav_executor.py): the batched
streaming vocoder of this package."""
from __future__ import annotations

from ..pipeline.stages import Code2WavStreamingExecutor, _device


def create_code2wav_executor(model_path: str = "", device: str = "cuda", chunk: int = 10, left_context: int = 25,
                             first_chunk: int | None = None, overrides: dict | None = None, **_):
    return Code2WavStreamingExecutor(model_path, _device(device), chunk, left_context, first_chunk, overrides)
