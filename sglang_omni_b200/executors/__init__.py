from .direct_model_executor import DirectModelExecutor
from .engine_executor import EngineExecutor
from .fused_executor import FusedExecutor, create_fused_executor
from .interface import Executor
from .preprocessing_executor import PreprocessingExecutor, StageError

__all__ = ["DirectModelExecutor", "EngineExecutor", "FusedExecutor", "create_fused_executor", "Executor",
           "PreprocessingExecutor", "StageError"]
