"""Fan-in of the encoder outputs into the thinker input (reference:
sglang_omni/models/qwen3_omni/pipeline/merge.py:41-316)."""
from __future__ import annotations

from ....proto import StagePayload


def merge_for_thinker(payloads: dict[str, StagePayload]) -> StagePayload:
    pre = payloads["preprocessing"]
    data = dict(pre.data)
    data.pop("audio_waveforms", None)
    data.pop("images", None)
    aud = payloads.get("audio_encoder")
    img = payloads.get("image_encoder")
    data["audio_embeds"] = (aud.data or {}).get("audio_embeds") if aud is not None and aud.data else None
    if img is not None and img.data:
        data["image_embeds"] = img.data.get("image_embeds")
        data["deepstack"] = img.data.get("deepstack")
    return StagePayload(pre.request_id, pre.request, data)
