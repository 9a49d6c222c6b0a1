"""Media inputs on CPU: video decode (OpenCV) and 2 fps frame sampling, URL / file /
data-URI fetching with a local HTTP server, WAV decode + polyphase resampling, and a
video + audio chat request through the tiny Qwen3-Omni text pipeline."""
import asyncio
import base64
import http.server
import io
import threading

import numpy as np
import pytest
import torch

from sglang_omni_b200.preprocessing import media


def _write_video(path, n=20, fps=10, hw=(48, 64)):
    import cv2

    w = cv2.VideoWriter(str(path), cv2.VideoWriter_fourcc(*"MJPG"), fps, (hw[1], hw[0]))
    for i in range(n):
        w.write(np.full((hw[0], hw[1], 3), (i * 12) % 255, np.uint8))
    w.release()


def _serve(directory):
    class H(http.server.SimpleHTTPRequestHandler):
        def __init__(self, *a, **k):
            super().__init__(*a, directory=str(directory), **k)

        def log_message(self, *a):
            pass

    srv = http.server.ThreadingHTTPServer(("127.0.0.1", 0), H)
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv


def test_video_decode_sampling_and_url(tmp_path):
    _write_video(tmp_path / "clip.avi")           # 2 s at 10 fps
    v = media.load_video(str(tmp_path / "clip.avi"))
    assert v["frames"].shape[0] == 4 and v["frames"].shape[1:] == (48, 64, 3)   # 2 fps, even count
    assert v["second_per_grid"] == 1.0
    srv = _serve(tmp_path)
    try:
        url = f"http://127.0.0.1:{srv.server_address[1]}/clip.avi"
        v2 = media.load_video(url)
        assert np.array_equal(v2["frames"], v["frames"])
        assert media.fetch(url) is media.fetch(url)      # cached by URL
    finally:
        srv.shutdown()
    arr = np.zeros((7, 32, 32, 3), np.uint8)
    v3 = media.load_video({"frames": arr, "fps": 2.0})
    assert v3["frames"].shape[0] == 8                    # padded to the temporal patch


def test_audio_wav_decode_and_resample(tmp_path):
    from scipy.io import wavfile

    sr = 22050
    x = (np.sin(np.arange(sr) * 2 * np.pi * 440 / sr) * 0.5).astype(np.float32)
    wavfile.write(tmp_path / "a.wav", sr, x)
    y = media.load_audio(str(tmp_path / "a.wav"))
    assert abs(y.shape[0] - 16000) <= 1
    b64 = "data:audio/wav;base64," + base64.b64encode((tmp_path / "a.wav").read_bytes()).decode()
    assert np.allclose(media.load_audio(b64), y)
    with pytest.raises(ValueError, match="only WAV"):
        media.load_audio(b"ID3\x04not-a-wav")


def test_video_audio_chat_request_tiny_pipeline(tmp_path):
    from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
    from sglang_omni_b200.config import PipelineRunner, compile_pipeline
    from sglang_omni_b200.models.qwen3_omni.config import Qwen3OmniPipelineConfig, text_stages
    from test_qwen3_omni_pipeline import TINY

    ovr = dict(TINY)
    ovr["vision"] = {"depth": 2, "hidden_size": 32, "intermediate_size": 64, "num_heads": 2,
                     "num_position_embeddings": 64, "deepstack_visual_indexes": [0], "dtype": torch.float32}
    _write_video(tmp_path / "clip.avi", n=10, fps=5, hw=(64, 64))
    cfg = Qwen3OmniPipelineConfig(model_path="random", stages=text_stages(overrides=ovr, device="cpu", max_batch=2,
                                                                          max_context=1024))

    async def main():
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            client = Client(coord)
            audio = (np.random.default_rng(1).standard_normal(16000) * 0.1).astype(np.float32)
            req = GenerateRequest(prompt="what is shown and heard?", videos=[str(tmp_path / "clip.avi")],
                                  audios=[audio], max_tokens=4, sampling=SamplingParams(temperature=0.0,
                                                                                        ignore_eos=True))
            return await client.completion(req)

    res = asyncio.run(main())
    assert len(res.token_ids) == 4
