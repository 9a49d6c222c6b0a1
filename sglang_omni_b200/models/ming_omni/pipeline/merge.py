"""Fan-in of the Ming-Omni aggregate stage: prompt layout + audio embeddings."""
from __future__ import annotations

from ....proto import StagePayload


def merge_for_thinker(payloads: dict[str, StagePayload]) -> StagePayload:
    pre = payloads["preprocessing"]
    data = dict(pre.data)
    data.pop("audio_waveforms", None)
    aud = payloads.get("audio_encoder")
    data["audio_embeds"] = (aud.data or {}).get("audio_embeds") if aud is not None and aud.data else None
    return StagePayload(pre.request_id, pre.request, data)
