"""Qwen3-Omni speech-in / speech-out in one process on one GPU: a WAV question in, the streamed
answer text printed, the streamed audio chunks written to a WAV file.

    python examples/qwen3_omni_speech.py --model-path <checkpoint or random> --audio question.wav
"""
import argparse
import asyncio
import time

import numpy as np

from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
from sglang_omni_b200.client.audio import encode_audio
from sglang_omni_b200.config import PipelineRunner, compile_pipeline
from sglang_omni_b200.models.qwen3_omni.config import Qwen3OmniPipelineConfig, text_stages


async def main(args):
    cfg = Qwen3OmniPipelineConfig(model_path=args.model_path,
                                  stages=text_stages(device="cuda:0", max_batch=8, speech=True, first_chunk=2))
    audio = args.audio or {"array": (np.random.default_rng(0).standard_normal(16000 * 5) * 0.1).astype(np.float32),
                           "sampling_rate": 16000}
    coord, stages = compile_pipeline(cfg)
    async with PipelineRunner(coord, stages):
        client = Client(coord)
        req = GenerateRequest(prompt=args.prompt, audios=[audio], max_tokens=args.max_tokens, stream=True,
                              sampling=SamplingParams(temperature=0.0), output_modalities=["text", "audio"])
        t0, first_audio, pcm, rate = time.perf_counter(), None, [], 24000
        async for ch in client.generate(req):
            if ch.modality == "audio" and ch.audio_data is not None and ch.finish_reason is None:
                first_audio = first_audio or time.perf_counter() - t0
                pcm.append(np.asarray(ch.audio_data, dtype=np.float32))
                rate = ch.sample_rate or rate
            elif ch.text and ch.finish_reason is None:
                print(ch.text, end="", flush=True)
        print()
    if pcm:
        with open(args.out, "wb") as f:
            f.write(encode_audio(np.concatenate(pcm), rate, "wav"))
        print(f"first audio chunk after {1e3 * first_audio:.0f} ms; {sum(len(p) for p in pcm) / rate:.1f} s "
              f"of audio written to {args.out}")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--model-path", default="random")
    ap.add_argument("--audio", help="WAV file (default: 5 s of noise)")
    ap.add_argument("--prompt", default="Answer the question in the audio.")
    ap.add_argument("--max-tokens", type=int, default=64)
    ap.add_argument("--out", default="answer.wav")
    asyncio.run(main(ap.parse_args()))
