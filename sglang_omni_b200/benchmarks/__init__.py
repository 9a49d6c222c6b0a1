"""Online serving benchmarks against a running server's HTTP API (this package's or any
server with the same OpenAI-compatible routes).

    python -m sglang_omni_b200.benchmarks tts-speed  --base-url http://127.0.0.1:8000 --concurrency 1,4,16
    python -m sglang_omni_b200.benchmarks omni-speed --base-url ... --stream
    python -m sglang_omni_b200.benchmarks tts-wer    --base-url ... --testset meta.lst --asr-model <whisper dir>

Counterpart of the reference's ``benchmarks/`` tree (benchmarker/runner.py, metrics/performance.py,
tasks/tts_speed.py, tasks/voice_clone.py, dataset/seedtts.py, eval/*.py): the same request
shapes, the same summary metrics (latency mean / median / p95 / p99, RTF, QPS, aggregate
tok/s = completion tokens / engine seconds) and the seed-tts-eval ``meta.lst`` input format, so
numbers from either tool compare.  Streamed requests also report time to first audio.
"""
from .datasets import SpeechSample, load_meta_lst, synthetic_samples
from .results import RequestOutcome, regression_failures, summarize
from .runner import run_requests

__all__ = ["SpeechSample", "load_meta_lst", "synthetic_samples", "RequestOutcome", "summarize",
           "regression_failures", "run_requests"]
