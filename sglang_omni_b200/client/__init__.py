from .audio import audio_to_base64, encode_audio
from .client import Client
from .types import (AbortLevel, AbortResult, ClientError, CompletionResult, CompletionStreamChunk, GenerateChunk,
                    GenerateRequest, Message, SpeechResult, UsageInfo)
from ..sampling_params import SamplingParams

__all__ = ["audio_to_base64", "encode_audio", "Client", "AbortLevel", "AbortResult", "ClientError",
           "CompletionResult", "CompletionStreamChunk", "GenerateChunk", "GenerateRequest", "Message",
           "SpeechResult", "UsageInfo", "SamplingParams"]
