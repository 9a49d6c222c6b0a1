"""The ``code_predictor`` stage of the reference's 9-stage speech layout
(sglang_omni/models/qwen3_omni/components/code_predictor_executor.py).

Here the code predictor runs inside the talker stage (one CUDA graph per frame:
talker step + 15 code-predictor steps), so this stage only forwards the talker's
code frames to code2wav: through the in-process fast lane when code2wav shares
the process, else over the relay.  The reference's feedback stream back to the
talker (bootstrap=False) carries nothing here: the talker already has every
code group of its frames.
"""
from __future__ import annotations

import asyncio

from ....executors.interface import Executor, ResultQueueMixin
from ....pipeline import fastlane
from ....proto import StagePayload
from ..pipeline.next_stage import CODE2WAV_STAGE, CODE_PREDICTOR_STAGE


class CodeFrameForwarder(ResultQueueMixin, Executor):
    def __init__(self, target: str = CODE2WAV_STAGE, stage_name: str = CODE_PREDICTOR_STAGE):
        super().__init__()
        self.target = target
        self.stage_name = stage_name

    async def start(self):
        fastlane.register(self.stage_name, self)

    async def stop(self):
        fastlane.unregister(self.stage_name, self)

    def deliver_many(self, items):
        lane = fastlane.get(self.target)
        if lane is not None:
            lane.deliver_many(items)
        elif self._stream_fn is not None:
            for rid, data in items:
                self._stream_fn(rid, data, self.target)

    async def add_request(self, payload: StagePayload) -> None:
        asyncio.ensure_future(self._pump(payload))

    async def _pump(self, payload: StagePayload):
        rid = payload.request_id
        frames = 0
        try:
            while True:
                item = await self._mailbox.get(rid)
                if item is None:
                    break
                if item.data.get("codes"):
                    frames += 1
                self._stream_fn(rid, item.data, self.target)
        except Exception as exc:  # the talker's stream failed
            from ....executors.preprocessing_executor import StageError

            self._results().put_nowait(StageError(rid, f"code_predictor: {exc}"))
            return
        self._results().put_nowait(StagePayload(rid, payload.request, {"num_frames": frames}))


def create_code_predictor_executor_from_config(model_path: str = "", code_predictor_max_seq_len: int = 256, **_):
    return CodeFrameForwarder()
