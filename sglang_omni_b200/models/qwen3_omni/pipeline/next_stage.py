"""Stage routing of the Qwen3-Omni pipelines (stage names as in
sglang_omni/models/qwen3_omni/pipeline/next_stage.py:11-92)."""
from __future__ import annotations

PREPROCESSING_STAGE = "preprocessing"
IMAGE_STAGE = "image_encoder"
AUDIO_STAGE = "audio_encoder"
AGGREGATE_STAGE = "mm_aggregate"
THINKER_STAGE = "thinker"
DECODE_STAGE = "decode"
TALKER_AR_STAGE = "talker_ar"
CODE_PREDICTOR_STAGE = "code_predictor"
CODE2WAV_STAGE = "code2wav"


def preprocessing_next(request_id, payload):
    return [IMAGE_STAGE, AUDIO_STAGE, AGGREGATE_STAGE]


def encoder_next(request_id, payload):
    return AGGREGATE_STAGE


def aggregate_next(request_id, payload):
    return THINKER_STAGE


def thinker_next(request_id, payload):
    return DECODE_STAGE


def decode_next(request_id, payload):
    return None


def talker_next(request_id, payload):
    return None


def code2wav_next(request_id, payload):
    return None


# names of the reference's 9-stage speech layout (talker_ar -> code_predictor -> code2wav)
def thinker_next_speech(request_id, payload):
    return DECODE_STAGE


def talker_ar_next(request_id, payload):
    return None


def code_predictor_next(request_id, payload):
    return None
