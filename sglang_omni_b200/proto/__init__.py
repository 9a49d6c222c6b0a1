from .messages import (AbortMessage, CompleteMessage, DataReadyMessage, ProfilerStartMessage, ProfilerStopMessage,
                       ShutdownMessage, StageStatsMessage, StreamMessage, SubmitMessage, parse_message)
from .request import OmniRequest, RequestInfo, RequestState, StagePayload
from .stage import StageInfo

__all__ = ["AbortMessage", "CompleteMessage", "DataReadyMessage", "ProfilerStartMessage", "ProfilerStopMessage",
           "ShutdownMessage", "StageStatsMessage", "StreamMessage", "SubmitMessage", "parse_message", "OmniRequest", "RequestInfo",
           "RequestState", "StagePayload", "StageInfo"]
