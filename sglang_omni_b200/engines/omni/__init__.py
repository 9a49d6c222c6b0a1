from .engine import OmniEngine
from .factory import create_ar_engine, create_encoder_engine
from .scheduler import Scheduler
from .types import ModelRunnerOutput, RequestOutput, SchedulerOutput, SchedulerRequest, SchedulerStatus

__all__ = ["OmniEngine", "create_ar_engine", "create_encoder_engine", "Scheduler", "ModelRunnerOutput",
           "RequestOutput", "SchedulerOutput", "SchedulerRequest", "SchedulerStatus"]
