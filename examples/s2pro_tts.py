"""S2-Pro-style streaming text-to-speech in one process: text in, 44.1 kHz audio streamed in
chunks, written to a WAV file; prints the time to the first chunk and the real-time factor.

    python examples/s2pro_tts.py --model-path <S2-Pro checkpoint or random> --text "Hello there."
"""
import argparse
import asyncio
import time

import numpy as np

from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
from sglang_omni_b200.client.audio import encode_audio
from sglang_omni_b200.config import PipelineRunner, compile_pipeline
from sglang_omni_b200.models.fishaudio_s2_pro.config import S2ProPipelineConfig, s2pro_stages


async def main(args):
    cfg = S2ProPipelineConfig(model_path=args.model_path,
                              stages=s2pro_stages(device="cuda:0", max_new_tokens=args.max_frames, max_streams=4))
    coord, stages = compile_pipeline(cfg)
    async with PipelineRunner(coord, stages):
        client = Client(coord)
        req = GenerateRequest(prompt=args.text, max_tokens=args.max_frames, output_modalities=["audio"], task="tts",
                              stream=True, sampling=SamplingParams(temperature=0.8, top_p=0.8, top_k=30))
        t0, first, pcm, rate = time.perf_counter(), None, [], 44100
        async for ch in client.generate(req):
            if ch.finish_reason is None and ch.modality == "audio" and ch.audio_data is not None:
                first = first or time.perf_counter() - t0
                pcm.append(np.asarray(ch.audio_data, dtype=np.float32))
                rate = ch.sample_rate or rate
        wall = time.perf_counter() - t0
    audio = np.concatenate(pcm) if pcm else np.zeros(0, np.float32)
    with open(args.out, "wb") as f:
        f.write(encode_audio(audio, rate, "wav"))
    secs = audio.size / rate
    print(f"{secs:.1f} s of audio to {args.out}; first chunk after {1e3 * (first or 0):.0f} ms; "
          f"real-time factor {wall / max(secs, 1e-9):.3f}")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--model-path", default="random")
    ap.add_argument("--text", default="Streaming speech synthesis on one GPU.")
    ap.add_argument("--max-frames", type=int, default=200, help="audio frames of 2048 samples at 44.1 kHz")
    ap.add_argument("--out", default="speech.wav")
    asyncio.run(main(ap.parse_args()))
