"""Smallest pipeline end to end on the CPU: an identity preprocessing stage feeding a 2-layer
decoder stage; four concurrent streaming requests through the in-process client.

    python examples/two_stage_toy.py
"""
import asyncio

from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
from sglang_omni_b200.config import PipelineRunner, compile_pipeline
from sglang_omni_b200.models.toy.config import ToyPipelineConfig


async def main():
    coord, stages = compile_pipeline(ToyPipelineConfig())
    async with PipelineRunner(coord, stages):
        client = Client(coord)

        async def one(i):
            req = GenerateRequest(prompt_token_ids=[(7 * i + j) % 1000 for j in range(32)], max_tokens=16,
                                  sampling=SamplingParams(temperature=0.0), stream=True)
            toks = []
            async for ch in client.generate(req):
                toks += ch.token_ids if ch.finish_reason is None else []
            return toks

        for i, toks in enumerate(await asyncio.gather(*[one(i) for i in range(4)])):
            print(f"request {i}: {toks}")


if __name__ == "__main__":
    asyncio.run(main())
