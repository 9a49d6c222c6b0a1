"""Stage load reports: every stage sends its queue depth and engine counters to the coordinator
periodically; /metrics returns the latest report of each stage (JSON and Prometheus gauges), and
the paged AR engine's report carries its KV-cache occupancy."""
import asyncio

import httpx

from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
from sglang_omni_b200.config import PipelineRunner, compile_pipeline
from sglang_omni_b200.models.toy.config import ToyPipelineConfig
from sglang_omni_b200.proto import StageStatsMessage, parse_message
from sglang_omni_b200.serve.openai_api import create_app


def test_stats_message_round_trip():
    m = parse_message(StageStatsMessage("decoder", {"queue_depth": 2, "kv_usage": 0.5}).to_dict())
    assert isinstance(m, StageStatsMessage) and m.stage == "decoder" and m.stats["kv_usage"] == 0.5


def test_stage_reports_reach_metrics(monkeypatch):
    monkeypatch.setenv("OMNI_STAGE_STATS_S", "0.05")

    async def main():
        coord, stages = compile_pipeline(ToyPipelineConfig())
        async with PipelineRunner(coord, stages):
            client = Client(coord)
            req = GenerateRequest(prompt_token_ids=[1, 2, 3], max_tokens=6,
                                  sampling=SamplingParams(temperature=0.0, ignore_eos=True))
            await client.completion(req)
            await asyncio.sleep(0.3)
            app = create_app(client, "toy")
            async with httpx.AsyncClient(transport=httpx.ASGITransport(app=app), base_url="http://t") as http:
                js = (await http.get("/metrics")).json()
                prom = (await http.get("/metrics", params={"format": "prometheus"})).text
            return js, prom, coord.health()

    js, prom, health = asyncio.run(main())
    st = js["stages"]
    assert set(st) == {"preprocessing", "decoder"}
    dec = st["decoder"]
    assert dec["queue_depth"] == 0 and dec["messages"] >= 1 and dec["age_s"] < 5
    assert dec["kv_pages_total"] > 0 and 0 <= dec["kv_usage"] <= 1 and dec["requests_running"] == 0
    assert dec["steps"] >= 6 and dec["step_ms"] > 0           # prefill + decode steps of the request
    assert 'omni_stage_kv_pages_total{stage="decoder"}' in prom and "# TYPE omni_stage_queue_depth gauge" in prom
    assert health["stage_stats"]["decoder"]["kv_pages_total"] == dec["kv_pages_total"]
