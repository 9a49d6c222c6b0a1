"""Two-stage CPU toy pipeline end to end: scheduler, relay, stream queue,
coordinator, client and the OpenAI server (8 concurrent requests x 32 prompt
ids, greedy 16 tokens, streaming)."""
import asyncio
import json

import httpx
import pytest
import torch

from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
from sglang_omni_b200.config import PipelineRunner, compile_pipeline
from sglang_omni_b200.models.toy.config import ToyPipelineConfig
from sglang_omni_b200.serve.openai_api import create_app


def _prompts(n=8, L=32):
    g = torch.Generator().manual_seed(0)
    return torch.randint(0, 1000, (n, L), generator=g).tolist()


def test_toy_pipeline_client_stream_and_batch():
    async def main():
        cfg = ToyPipelineConfig()
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            client = Client(coord)
            prompts = _prompts()

            async def one(i):
                req = GenerateRequest(prompt_token_ids=prompts[i], sampling=SamplingParams(temperature=0.0),
                                      max_tokens=16, stream=True)
                toks, final = [], None
                async for ch in client.generate(req):
                    if ch.finish_reason is None:
                        toks += ch.token_ids
                    else:
                        final = ch
                return toks, final

            outs = await asyncio.gather(*[one(i) for i in range(8)])
            for toks, final in outs:
                assert len(toks) == 16
                assert final.usage.completion_tokens == 16 and final.usage.prompt_tokens == 32
                assert final.token_ids == toks
            # non-streaming agrees with streaming (greedy, deterministic)
            res = await client.completion(GenerateRequest(prompt_token_ids=prompts[0], max_tokens=16,
                                                          sampling=SamplingParams(temperature=0.0)))
            assert res.token_ids == outs[0][0]
            assert coord.health()["requests"]["completed"] >= 9

    asyncio.run(main())


def test_toy_pipeline_openai_server_sse():
    async def main():
        cfg = ToyPipelineConfig()
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            app = create_app(Client(coord), "toy")
            transport = httpx.ASGITransport(app=app)
            async with httpx.AsyncClient(transport=transport, base_url="http://t") as http:
                r = await http.get("/health")
                assert r.status_code == 200
                r = await http.get("/v1/models")
                assert r.json()["data"][0]["id"] == "toy"
                r = await http.get("/playground")
                assert r.status_code == 200 and "/v1/chat/completions" in r.text
                prompts = _prompts()

                async def chat(i, stream):
                    body = {"messages": [{"role": "user", "content": "x"}], "prompt_token_ids": prompts[i],
                            "max_tokens": 16, "temperature": 0.0, "stream": stream}
                    r = await http.post("/v1/chat/completions", json=body)
                    assert r.status_code == 200
                    if not stream:
                        return r.json()
                    events = [ln[6:] for ln in r.text.splitlines() if ln.startswith("data: ")]
                    assert events[-1] == "[DONE]"
                    chunks = [json.loads(e) for e in events[:-1]]
                    assert chunks[0]["choices"][0]["delta"]["role"] == "assistant"
                    assert chunks[-1]["choices"][0]["finish_reason"] == "length"
                    assert chunks[-1]["usage"]["completion_tokens"] == 16
                    return chunks

                outs = await asyncio.gather(*[chat(i, True) for i in range(8)])
                assert len(outs) == 8
                full = await chat(0, False)
                assert full["usage"]["completion_tokens"] == 16
                assert full["choices"][0]["message"]["role"] == "assistant"
                m = (await http.get("/metrics")).json()
                assert m["requests_ok"] == 9 and m["requests_in_flight"] == 0 and m["completion_tokens"] == 144
                assert m["ttft_p50_s"] is not None and m["itl_p50_s"] is not None
                prom = (await http.get("/metrics", params={"format": "prometheus"})).text
                assert 'omni_requests_total{status="ok"} 9' in prom
                assert 'omni_time_to_first_token_seconds{quantile="0.5"}' in prom

    asyncio.run(main())


def test_toy_pipeline_abort():
    async def main():
        cfg = ToyPipelineConfig()
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            client = Client(coord)
            req = GenerateRequest(prompt_token_ids=_prompts(1)[0], max_tokens=200,
                                  sampling=SamplingParams(temperature=0.0, ignore_eos=True), request_id="ab1",
                                  stream=False)
            task = asyncio.ensure_future(client.completion(req))
            await asyncio.sleep(0.05)
            await client.abort("ab1")
            with pytest.raises(asyncio.CancelledError):
                await task
            # the pipeline still serves after an abort
            res = await client.completion(GenerateRequest(prompt_token_ids=_prompts(1)[0], max_tokens=4,
                                                          sampling=SamplingParams(temperature=0.0)))
            assert len(res.token_ids) == 4

    asyncio.run(main())


def test_toy_pipeline_under_asyncio_debug_mode():
    """The event-loop side of the runtime under asyncio's debug mode: no coroutine is left
    un-awaited, no callback is scheduled from a foreign thread without the thread-safe entry
    point (debug mode raises for that), no task dies with an unretrieved exception, and the
    pipeline still completes every request."""
    import gc
    import logging
    import warnings

    records = []

    class _Grab(logging.Handler):
        def emit(self, rec):
            records.append(rec.getMessage())

    h = _Grab(level=logging.ERROR)
    logging.getLogger("asyncio").addHandler(h)

    async def main():
        loop = asyncio.get_running_loop()
        loop.slow_callback_duration = 10.0   # timing is not under test here
        cfg = ToyPipelineConfig()
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            client = Client(coord)
            prompts = _prompts(4)

            async def one(i):
                req = GenerateRequest(prompt_token_ids=prompts[i], sampling=SamplingParams(temperature=0.0),
                                      max_tokens=8, stream=True)
                n = 0
                async for ch in client.generate(req):
                    n += len(ch.token_ids) if ch.finish_reason is None else 0
                return n

            assert await asyncio.gather(*[one(i) for i in range(4)]) == [8] * 4

    try:
        with warnings.catch_warnings(record=True) as w:
            warnings.simplefilter("always")
            asyncio.run(main(), debug=True)
            gc.collect()
        never = [str(x.message) for x in w if "was never awaited" in str(x.message)]
        assert not never, never
        bad = [m for m in records if "exception was never retrieved" in m or "non-thread-safe" in m]
        assert not bad, bad
    finally:
        logging.getLogger("asyncio").removeHandler(h)
