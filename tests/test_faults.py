"""Host-side fault injection through the control plane (no GPU involved).

Against the CPU toy pipeline (in-process and with one OS process per stage over
ZMQ + shared memory):
* a dropped completion runs into the coordinator's request deadline and fails
  only that request; the next requests still complete;
* duplicated stream chunks are dropped by their sequence numbers (the client
  sees every token once);
* delayed messages only delay;
* a corrupted relay descriptor (shared-memory segment / offsets that do not
  exist) fails that request at the receiving stage, and the pipeline keeps
  serving.
"""
import asyncio

import pytest
import torch

from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
from sglang_omni_b200.config import PipelineRunner, compile_pipeline
from sglang_omni_b200.models.toy.config import ToyPipelineConfig
from sglang_omni_b200.pipeline import faults
from sglang_omni_b200.pipeline.faults import FaultRule


@pytest.fixture(autouse=True)
def _clean():
    faults.clear()
    yield
    faults.clear()


def _prompt(i, L=20):
    return torch.randint(0, 1000, (L,), generator=torch.Generator().manual_seed(100 + i)).tolist()


async def _stream(client, i, n=8):
    req = GenerateRequest(prompt_token_ids=_prompt(i), sampling=SamplingParams(temperature=0.0), max_tokens=n,
                          stream=True)
    toks = []
    async for ch in client.generate(req):
        if ch.finish_reason is None:
            toks += ch.token_ids
    return toks


def _run(cfg, body):
    async def main():
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            return await body(Client(coord))

    return asyncio.run(main())


def test_dropped_completion_fails_by_deadline_then_pipeline_recovers():
    ref = _run(ToyPipelineConfig(), lambda c: _stream(c, 0))
    faults.inject([FaultRule("drop", "complete", from_stage="decoder", count=1)])
    cfg = ToyPipelineConfig(request_timeout_s=2.0)

    async def body(client):
        with pytest.raises(Exception, match="did not complete"):
            await asyncio.wait_for(_stream(client, 0), timeout=30)
        return await asyncio.wait_for(_stream(client, 0), timeout=30)

    assert _run(cfg, body) == ref


def test_duplicated_and_delayed_chunks():
    ref = _run(ToyPipelineConfig(), lambda c: asyncio.gather(*[_stream(c, i) for i in range(3)]))
    faults.inject([FaultRule("duplicate", "stream", count=-1), FaultRule("delay", "data_ready", count=-1,
                                                                         delay_s=0.02)])
    out = _run(ToyPipelineConfig(), lambda c: asyncio.gather(*[_stream(c, i) for i in range(3)]))
    assert out == ref


def test_corrupted_relay_metadata_fails_one_request_multiprocess():
    """One OS process per stage: the preprocessing -> decoder hand-off goes through shared
    memory; its descriptor is corrupted once, in the sending stage process."""
    from sglang_omni_b200.pipeline.mp_runner import MultiProcessPipelineRunner

    cfg = ToyPipelineConfig(relay_backend="shm", request_timeout_s=60.0)
    cfg.stages[0].executor.args["inject_faults"] = [{"action": "corrupt", "kind": "data_ready", "count": 1}]

    async def main():
        runner = MultiProcessPipelineRunner(cfg, startup_timeout=120, monitor_interval=0.5)
        await runner.start()
        try:
            client = Client(runner.coordinator)
            with pytest.raises(Exception):
                await asyncio.wait_for(_stream(client, 1), timeout=60)
            return await asyncio.wait_for(_stream(client, 1), timeout=60)
        finally:
            await runner.stop()

    ref = _run(ToyPipelineConfig(), lambda c: _stream(c, 1))
    assert asyncio.run(main()) == ref
