"""Stage addressing record (sglang_omni/proto/stage.py:6)."""
from dataclasses import dataclass


@dataclass
class StageInfo:
    name: str
    control_endpoint: str
