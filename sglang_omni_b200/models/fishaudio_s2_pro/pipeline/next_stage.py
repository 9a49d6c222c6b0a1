"""Stage routing of the S2-Pro TTS pipeline (stage names as in
sglang_omni/models/fishaudio_s2_pro/pipeline/next_stage.py:9-25)."""
from __future__ import annotations

PREPROCESSING_STAGE = "preprocessing"
TTS_ENGINE_STAGE = "tts_engine"
VOCODER_STAGE = "vocoder"


def preprocessing_next(request_id, output):
    return TTS_ENGINE_STAGE


def tts_engine_next(request_id, output):
    return VOCODER_STAGE


def vocoder_next(request_id, output):
    return None
