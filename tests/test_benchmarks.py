"""Serving benchmarks against a live HTTP server on the CPU: the S2-Pro TTS pipeline through
/v1/audio/speech (plain and streamed, several concurrency levels, WER with a stand-in ASR) and
the Qwen3-Omni speech pipeline through /v1/chat/completions; metric definitions and the
regression gate on hand-made outcomes."""
import asyncio
import json
import socket
import threading
import time

import httpx
import pytest
import torch

from sglang_omni_b200.benchmarks import RequestOutcome, regression_failures, summarize
from sglang_omni_b200.benchmarks.__main__ import main as bench_main
from sglang_omni_b200.benchmarks.datasets import load_meta_lst
from sglang_omni_b200.benchmarks.wer import align, score, wer_summary

S2_TINY = {
    "slow": {"vocab_size": 512, "hidden_size": 64, "num_layers": 2, "num_heads": 4, "num_kv_heads": 2,
             "head_dim": 64, "intermediate_size": 128},
    "fast": {"hidden_size": 64, "num_layers": 2, "num_heads": 4, "num_kv_heads": 2, "head_dim": 64,
             "intermediate_size": 128},
    "s2pro": {"codebook_size": 64, "num_codebooks": 4},
    "dac": dict(latent_dim=64, decoder_dim=128, tf_layers=2, tf_heads=1, tf_head_dim=64, tf_inter=128,
                tf_window=8, encoder_dim=8, encoder_transformer_layers=(0, 0, 0, 1), n_codebooks=3,
                codebook_size=32, semantic_codebook_size=64),
}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _Server:
    """A pipeline and its OpenAI app under uvicorn on a background thread."""

    def __init__(self, cfg, model_name):
        import uvicorn

        from sglang_omni_b200.client import Client
        from sglang_omni_b200.config import PipelineRunner, compile_pipeline
        from sglang_omni_b200.serve.openai_api import create_app

        self.port = _free_port()
        self.url = f"http://127.0.0.1:{self.port}"
        self.server = None

        async def run():
            coord, stages = compile_pipeline(cfg)
            async with PipelineRunner(coord, stages):
                app = create_app(Client(coord), model_name)
                self.server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=self.port,
                                                            log_level="warning"))
                await self.server.serve()

        self.thread = threading.Thread(target=lambda: asyncio.run(run()), daemon=True)
        self.thread.start()
        t0 = time.time()
        while True:
            try:
                if httpx.get(self.url + "/health", timeout=1.0).status_code == 200:
                    break
            except httpx.HTTPError:
                pass
            assert time.time() - t0 < 120, "server did not come up"
            time.sleep(0.2)

    def close(self):
        if self.server is not None:
            self.server.should_exit = True
        self.thread.join(60)


@pytest.fixture(scope="module")
def s2pro_server():
    from sglang_omni_b200.models.fishaudio_s2_pro.config import S2ProPipelineConfig, s2pro_stages

    cfg = S2ProPipelineConfig(model_path="random", stages=s2pro_stages(
        overrides=S2_TINY, device="cpu", max_new_tokens=6, max_streams=4, max_context=512, stream_stride=2,
        stream_followup_stride=2))
    srv = _Server(cfg, "s2-pro")
    yield srv
    srv.close()


def test_tts_speed_plain_and_streamed(s2pro_server, tmp_path):
    out = tmp_path / "res"
    for stream in (False, True):
        argv = ["tts-speed", "--base-url", s2pro_server.url, "--max-samples", "3", "--concurrency", "1,2",
                "--max-new-tokens", "6", "--output-dir", str(out), "--warmup", "1"] + (["--stream"] if stream else [])
        assert bench_main(argv) == 0
        res = json.loads((out / "tts-speed.json").read_text())
        assert [lv["concurrency"] for lv in res["levels"]] == [1, 2]
        for lv in res["levels"]:
            s = lv["summary"]
            assert s["completed_requests"] == 3 and s["failed_requests"] == 0, lv["outcomes"][0]["error"]
            assert s["rtf_mean"] > 0 and s["throughput_qps"] > 0 and s["audio_duration_mean_s"] > 0
            assert s["gen_tokens_total"] > 0 and s["tok_per_s_agg"] > 0
            if stream:
                assert s["ttfa_median_s"] <= s["latency_median_s"]
            # 44.1 kHz, whole code frames of 2048 samples
            for o in lv["outcomes"]:
                assert abs(o["audio_s"] * 44100 / 2048 - round(o["audio_s"] * 44100 / 2048)) < 1e-3


def test_tts_speed_regression_gate(s2pro_server, tmp_path):
    base = tmp_path / "base.json"
    base.write_text(json.dumps({"throughput_qps": 1e6}))      # unreachable: must fail the gate
    argv = ["tts-speed", "--base-url", s2pro_server.url, "--max-samples", "2", "--output-dir", str(tmp_path),
            "--max-new-tokens", "4", "--baseline", str(base)]
    assert bench_main(argv) == 1
    base.write_text(json.dumps({"1": {"latency_mean_s": 1e6}}))
    assert bench_main(argv) == 0


def fake_asr(wave, rate, lang):
    """Stand-in ASR: 'hears' the first synthetic sentence's words with one word dropped."""
    return "the quick brown"


def test_tts_wer_with_pluggable_asr(s2pro_server, tmp_path):
    meta = tmp_path / "meta.lst"
    meta.write_text("u1|ref one|wavs/u1.wav|The quick brown fox.\nu2||x.wav|Quick brown!\n")
    rows = load_meta_lst(str(meta))
    assert rows[0].ref_audio == str(tmp_path / "wavs" / "u1.wav") and rows[1].target_text == "Quick brown!"
    argv = ["tts-wer", "--base-url", s2pro_server.url, "--testset", str(meta), "--no-ref-audio",
            "--output-dir", str(tmp_path / "w"), "--max-new-tokens", "4", "--asr", f"{__name__}:fake_asr",
            "--warmup", "0"]
    assert bench_main(argv) == 0
    res = json.loads((tmp_path / "w" / "tts-wer.json").read_text())
    w = res["levels"][0]["wer"]
    # u1: 4 reference words, 1 deletion; u2: 2 words, 1 insertion ("the")
    assert w["evaluated"] == 2 and abs(w["wer_corpus"] - 2 / 6) < 1e-9
    assert res["levels"][0]["outcomes"][0]["asr_text"] == "the quick brown"


def test_omni_speed_chat_audio():
    from sglang_omni_b200.models.qwen3_omni.config import Qwen3OmniSpeechPipelineConfig, text_stages

    f32 = {"dtype": torch.float32}
    dec = {"num_layers": 2, "hidden_size": 64, "num_heads": 4, "num_kv_heads": 2, "head_dim": 32, **f32}
    tiny = {"thinker": {**dec, "num_experts": 8, "topk": 2, "moe_intermediate_size": 32, "mrope_section": [6, 5, 5]},
            "talker": {**dec, "num_experts": 8, "topk": 2, "moe_intermediate_size": 32,
                       "shared_expert_intermediate_size": 32, "intermediate_size": 64, "mrope_section": [6, 5, 5]},
            "code_predictor": {**dec, "num_layers": 1, "intermediate_size": 64},
            "audio": {"encoder_layers": 1, "encoder_attention_heads": 2, "encoder_ffn_dim": 64, "d_model": 64,
                      "downsample_hidden_size": 8, **f32},
            "code2wav": {"codebook_size": 2048, "hidden_size": 64, "num_heads": 4, "num_kv_heads": 4,
                         "intermediate_size": 64, "num_layers": 1, "upsample_rates": (2, 2),
                         "upsampling_ratios": (2,), "decoder_dim": 32, **f32}}
    cfg = Qwen3OmniSpeechPipelineConfig(model_path="random", stages=text_stages(
        overrides=tiny, device="cpu", max_batch=4, max_context=1024, speech=True, tail_frames=2, first_chunk=2))
    srv = _Server(cfg, "qwen3-omni")
    try:
        for stream in (False, True):
            out = {}
            import tempfile
            with tempfile.TemporaryDirectory() as d:
                argv = ["omni-speed", "--base-url", srv.url, "--max-samples", "2", "--concurrency", "2",
                        "--max-tokens", "4", "--output-dir", d, "--warmup", "0"] + (["--stream"] if stream else [])
                assert bench_main(argv) == 0
                with open(f"{d}/omni-speed.json") as f:
                    out = json.load(f)
            s = out["levels"][0]["summary"]
            assert s["completed_requests"] == 2, out["levels"][0]["outcomes"][0]["error"]
            assert s["audio_duration_mean_s"] > 0
            if stream:
                assert "ttfa_median_s" in s and "ttft_median_s" in s
    finally:
        srv.close()


def test_metrics_and_alignment_definitions():
    outs = [RequestOutcome("a", ok=True, latency_s=1.0, audio_s=2.0, completion_tokens=10, engine_time_s=0.5,
                           ttfa_s=0.2),
            RequestOutcome("b", ok=True, latency_s=3.0, audio_s=3.0, completion_tokens=30, engine_time_s=1.5),
            RequestOutcome("c", ok=False, error="boom")]
    s = summarize(outs, wall_s=4.0)
    assert s["completed_requests"] == 2 and s["failed_requests"] == 1
    assert s["latency_mean_s"] == 2.0 and s["rtf_mean"] == 0.75 and s["throughput_qps"] == 0.5
    assert s["tok_per_s_agg"] == 20.0 and s["audio_s_per_s"] == 1.25 and s["ttfa_median_s"] == 0.2
    assert regression_failures(s, {"throughput_qps": 0.6, "latency_mean_s": 1.7}) == []
    assert len(regression_failures(s, {"throughput_qps": 0.7, "latency_mean_s": 1.5, "rtf_mean": None})) == 2
    al = align("a b c d".split(), "a x c d e".split())
    assert (al.hits, al.substitutions, al.deletions, al.insertions) == (3, 1, 0, 1)
    assert score("Hello, World!", "hello world").rate == 0.0
    assert score("你好，世界", "你好世界", "zh").rate == 0.0
    summ = wer_summary([al, None, score("red blue", "red blue")])
    assert summ["evaluated"] == 2 and summ["skipped"] == 1 and abs(summ["wer_corpus"] - 2 / 6) < 1e-9
    assert summ["n_above_50_pct_wer"] == 0
