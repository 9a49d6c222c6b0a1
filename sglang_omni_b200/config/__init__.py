from .compiler import compile_pipeline
from .manager import ConfigManager
from .runner import PipelineRunner
from .schema import (EndpointsConfig, ExecutorConfig, InputHandlerConfig, PipelineConfig, RelayConfig, StageConfig,
                     StreamTargetConfig)

__all__ = ["compile_pipeline", "ConfigManager", "PipelineRunner", "EndpointsConfig", "ExecutorConfig",
           "InputHandlerConfig", "PipelineConfig", "RelayConfig", "StageConfig", "StreamTargetConfig"]
