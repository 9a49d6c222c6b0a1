"""Encoder runtime: batches up to ``max_batch_size`` requests per step.  Dict
inputs concatenate the ragged keys (pixel_values / input_features / grids /
lengths) and stack the rest; ``_skip`` requests (modality absent) bypass the
model; outputs are split back per request by the recorded row counts
(sglang_omni/engines/omni/runtime/encoder.py:19-526)."""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any

import torch

from ..types import ModelRunnerOutput, RequestOutput, SchedulerOutput

CAT_KEYS = ("pixel_values", "pixel_values_videos", "input_features", "image_grid_thw", "video_grid_thw",
            "feature_lens", "audio_feature_lengths", "patches", "grid_thw", "mel", "mel_lens")


@dataclass
class EncoderRequestData:
    inputs: dict[str, Any]
    skip: bool = False
    counts: dict[str, int] = field(default_factory=dict)
    cache_key: str | None = None      # media key from preprocessing: equal keys reuse one output


class EncoderBatchPlanner:
    """Up to ``max_batch_size`` waiting requests per step.  With ``gather_window_s``
    a partial batch waits until its oldest request has waited that long, so a
    burst of arrivals (requests leaving preprocessing a few ms apart) is encoded
    as one batch instead of a small batch followed by a large one."""

    def __init__(self, max_batch_size: int = 32, gather_window_s: float = 0.0):
        self.max_batch_size = max_batch_size
        self.gather_window_s = gather_window_s
        self._seen: dict[str, float] = {}

    def select_requests(self, waiting, running, resources):
        if self.gather_window_s > 0 and 0 < len(waiting) < self.max_batch_size:
            now = time.monotonic()
            first = min(self._seen.setdefault(r.request_id, now) for r in waiting)
            if now - first < self.gather_window_s:
                return []
        for r in waiting[: self.max_batch_size]:
            self._seen.pop(r.request_id, None)
        out = []
        for r in waiting:
            if len(out) >= self.max_batch_size or not resources.can_allocate(r):
                break
            out.append(r)
        return out

    def build_batch(self, requests):
        return [r.data for r in requests]


class EncoderInputPreparer:
    def prepare(self, sched_out: SchedulerOutput, device) -> dict[str, Any]:
        items = [r.data for r in sched_out.requests if not getattr(r.data, "skip", False)]
        if not items:
            return {"_empty": True}
        keys = items[0].inputs.keys()
        out: dict[str, Any] = {}
        for k in keys:
            vals = [it.inputs[k] for it in items]
            if isinstance(vals[0], torch.Tensor):
                if k in CAT_KEYS or vals[0].dim() == 0 or any(v.shape != vals[0].shape for v in vals):
                    out[k] = torch.cat([v.reshape(-1, *v.shape[1:]) if v.dim() else v.reshape(1) for v in vals])
                else:
                    out[k] = torch.stack(vals)
                out[k] = out[k].to(device, non_blocking=True)
            else:
                out[k] = vals
        out["_batch_sizes"] = [int(it.counts.get("rows", 1)) for it in items]
        return out


class EncoderOutputProcessor:
    """Splits the batched output rows back per request by ``counts['out_rows']``."""

    def process(self, model_output, sched_out: SchedulerOutput) -> ModelRunnerOutput:
        outs = {}
        reqs = [r for r in sched_out.requests if not getattr(r.data, "skip", False)]
        if isinstance(model_output, dict) and "_per_request" in model_output:
            per = model_output["_per_request"]
        else:
            sizes = [int(r.data.counts.get("out_rows", 1)) for r in reqs]
            per = list(torch.split(model_output, sizes)) if isinstance(model_output, torch.Tensor) else model_output
        for r, o in zip(reqs, per):
            outs[r.request_id] = RequestOutput(r.request_id, o, finished=True)
        for r in sched_out.requests:
            if getattr(r.data, "skip", False):
                outs[r.request_id] = RequestOutput(r.request_id, None, finished=True)
        return ModelRunnerOutput(outs, [r.request_id for r in sched_out.requests])


class EncoderModelWrapper:
    """Adapts ``encoder(batch_inputs) -> list per request`` to the generic runner's model(**inputs)."""

    def __init__(self, fn):
        self.fn = fn

    def __call__(self, **inputs):
        if inputs.get("_empty"):
            return {"_per_request": []}
        return {"_per_request": self.fn(inputs)}
