"""Multi-process pipeline (one process per stage, shm relay) on CPU, and
failure detection when a stage process dies (host-side fault, no GPU)."""
import asyncio
import os
import signal

import pytest

from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
from sglang_omni_b200.models.toy.config import ToyPipelineConfig
from sglang_omni_b200.pipeline.mp_runner import MultiProcessPipelineRunner


def test_mp_runner_toy_pipeline():
    async def main():
        cfg = ToyPipelineConfig(relay_backend="shm")
        async with MultiProcessPipelineRunner(cfg, startup_timeout=120, monitor_interval=0.5) as runner:
            client = Client(runner.coordinator)
            outs = await asyncio.gather(*[
                client.completion(GenerateRequest(prompt_token_ids=list(range(i, i + 32)), max_tokens=8,
                                                  sampling=SamplingParams(temperature=0.0))) for i in range(4)])
            assert all(len(o.token_ids) == 8 for o in outs)

    asyncio.run(main())


def test_mp_runner_detects_dead_stage():
    async def main():
        cfg = ToyPipelineConfig(relay_backend="shm")
        runner = MultiProcessPipelineRunner(cfg, startup_timeout=120, monitor_interval=0.2)
        await runner.start()
        try:
            client = Client(runner.coordinator)
            # kill the decoder stage process mid-flight
            os.kill(runner.procs[1].pid, signal.SIGKILL)
            req = GenerateRequest(prompt_token_ids=list(range(32)), max_tokens=400,
                                  sampling=SamplingParams(temperature=0.0, ignore_eos=True))
            with pytest.raises(Exception):
                await asyncio.wait_for(client.completion(req), timeout=20)
            await asyncio.sleep(0.5)
            assert runner.failed_stage == "decoder"
            assert not runner.coordinator.running
        finally:
            await runner.stop()

    asyncio.run(main())


def test_mp_runner_restarts_a_dead_stage():
    """With restart on, a killed stage process is replaced on the same endpoints: the request in
    flight fails, later requests are served, and the pipeline keeps running."""
    async def main():
        cfg = ToyPipelineConfig(relay_backend="shm")
        runner = MultiProcessPipelineRunner(cfg, startup_timeout=120, monitor_interval=0.2, restart=["decoder"])
        await runner.start()
        try:
            client = Client(runner.coordinator)
            req = lambda n: GenerateRequest(prompt_token_ids=list(range(32)), max_tokens=n,  # noqa: E731
                                            sampling=SamplingParams(temperature=0.0, ignore_eos=True))
            first = await client.completion(req(8))
            assert runner.restartable("decoder") and not runner.restartable("preprocessing")
            old = runner.procs[1].pid
            os.kill(old, signal.SIGKILL)
            with pytest.raises(Exception):
                await asyncio.wait_for(client.completion(req(400)), timeout=60)
            for _ in range(600):
                if runner.restarts.get("decoder") == 1 and runner.procs[1].is_alive():
                    break
                await asyncio.sleep(0.1)
            assert runner.procs[1].pid != old and runner.coordinator.running and runner.failed_stage is None
            again = await asyncio.wait_for(client.completion(req(8)), timeout=120)
            assert again.token_ids == first.token_ids     # same weights (seeded) after the restart
        finally:
            await runner.stop()

    asyncio.run(main())
