"""Reference factory path of the Code2Wav stage
(sglang_omni/models/qwen3_omni/components/code2wav_executor.py:236-259): the
batched streaming vocoder of this package.  The reference's argument names map
onto it: ``stream_chunk_size`` -> chunk, ``left_context_size`` -> left context
(used by ``mode="window"``), ``max_batch_size`` -> largest graph batch,
``gpu_id`` -> device (unless a device other than "cuda" is given)."""
from __future__ import annotations

from ..pipeline.stages import Code2WavStreamingExecutor, _device


def create_code2wav_executor(model_path: str = "", device: str = "cuda", chunk: int | None = None,
                             left_context: int | None = None, first_chunk: int | None = None,
                             overrides: dict | None = None, *, stream_chunk_size: int = 10,
                             left_context_size: int = 25, max_batch_size: int = 32, gpu_id: int | None = None,
                             mode: str = "stateful", dtype: str | None = None, **_):
    if gpu_id is not None and device == "cuda":
        device = f"cuda:{gpu_id}"
    return Code2WavStreamingExecutor(model_path, _device(device), chunk or stream_chunk_size,
                                     left_context if left_context is not None else left_context_size, first_chunk,
                                     overrides, max_streams=max_batch_size, mode=mode)
