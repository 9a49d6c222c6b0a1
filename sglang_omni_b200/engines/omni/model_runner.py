"""Generic model runner: InputPreparer -> model(**inputs) under inference mode
-> OutputProcessor (sglang_omni/engines/omni/model_runner.py:19-77)."""
from __future__ import annotations

import torch


class ModelRunner:
    def __init__(self, model, input_preparer, output_processor, device="cpu"):
        self.model = model
        self.input_preparer = input_preparer
        self.output_processor = output_processor
        self.device = torch.device(device)

    def execute(self, sched_out):
        inputs = self.input_preparer.prepare(sched_out, self.device)
        with torch.inference_mode():
            out = self.model(**inputs)
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()
        return self.output_processor.process(out, sched_out)
