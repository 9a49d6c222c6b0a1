"""Stage routing of the Ming-Omni text and speech pipelines (stage names as in
sglang_omni/models/ming_omni/pipeline/next_stage.py:11-67)."""
from __future__ import annotations

PREPROCESSING_STAGE = "preprocessing"
AUDIO_STAGE = "audio_encoder"
AGGREGATE_STAGE = "mm_aggregate"
THINKER_STAGE = "thinker"
DECODE_STAGE = "decode"
TALKER_STAGE = "talker"


def preprocessing_next(request_id, output):
    return [AUDIO_STAGE, AGGREGATE_STAGE]


def encoder_next(request_id, output):
    return AGGREGATE_STAGE


def aggregate_next(request_id, output):
    return THINKER_STAGE


def thinker_next(request_id, output):
    return DECODE_STAGE


def thinker_next_speech(request_id, output):
    """Speech output: the thinker's result goes to decode (text) and to the talker."""
    return [DECODE_STAGE, TALKER_STAGE]


def decode_next(request_id, output):
    return None


def talker_next(request_id, output):
    return None
