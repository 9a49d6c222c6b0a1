"""Media cache keys and the encoder output caches they drive: content fingerprints of every
media form a request can carry, keys that change with the preprocessing context, and the
Qwen3-Omni audio / vision towers serving a repeated clip or image from their cache (same
thinker output, one encoder forward), with caching off when the pipeline asks for it."""
import asyncio
import os

import numpy as np
import pytest
import torch

from sglang_omni_b200.engines.omni.runtime.cache import SimpleCacheManager, cache_key_of
from sglang_omni_b200.engines.omni.runtime.encoder import EncoderRequestData
from sglang_omni_b200.preprocessing.cache_key import fingerprint, media_cache_key


def test_fingerprints_follow_content(tmp_path):
    a = np.arange(1000, dtype=np.float32)
    assert fingerprint(a) == fingerprint(a.copy()) != fingerprint(a[::-1].copy())
    assert fingerprint(a) != fingerprint(a.astype(np.float64))
    assert fingerprint(torch.from_numpy(a)) == fingerprint(torch.from_numpy(a).clone())
    f1, f2 = tmp_path / "x.wav", tmp_path / "y.wav"
    f1.write_bytes(b"RIFF" + bytes(5000))
    f2.write_bytes(b"RIFF" + bytes(2400) + b"\x01" + bytes(2599))     # differs only in the middle
    assert fingerprint(str(f1)) != fingerprint(str(f2))
    assert fingerprint(str(f1)) == fingerprint("file://" + str(f1))
    assert fingerprint("https://h/a.png") != fingerprint("https://h/b.png")
    assert fingerprint({"url": "https://h/a.png", "detail": 1}) == fingerprint({"detail": 1, "url": "https://h/a.png"})
    assert fingerprint(object()) is None
    k = media_cache_key("audio", [a], sample_rate=16000)
    assert k == media_cache_key("audio", [a.copy()], sample_rate=16000)
    assert k != media_cache_key("audio", [a], sample_rate=24000)
    assert k != media_cache_key("audio", [a, a], sample_rate=16000)
    assert media_cache_key("audio", []) is None and media_cache_key("audio", [a, object()]) is None


def test_cache_manager_explicit_keys():
    class R:
        def __init__(self, data):
            self.data = data

    m = SimpleCacheManager(2, explicit_only=True)
    keyed = R(EncoderRequestData(inputs={"x": torch.ones(3)}, cache_key="k1"))
    unkeyed = R(EncoderRequestData(inputs={"x": torch.ones(3)}))
    m.put(keyed, {"out": 1})
    m.put(unkeyed, {"out": 2})
    assert m.get(R(EncoderRequestData(inputs={}, cache_key="k1"))) == {"out": 1}
    assert m.get(unkeyed) is None and len(m._d) == 1
    # without explicit_only a dataclass request hashes its fields (tensors by content)
    assert cache_key_of(EncoderRequestData(inputs={"x": torch.ones(3)})) == \
        cache_key_of(EncoderRequestData(inputs={"x": torch.ones(3)}))
    assert cache_key_of(EncoderRequestData(inputs={"x": torch.ones(3)})) != \
        cache_key_of(EncoderRequestData(inputs={"x": torch.zeros(3)}))


def _engine_of(stages, name):
    for st in stages:
        if getattr(st, "name", None) == name:
            return st.workers[0].executor.engine
    raise KeyError(name)


@pytest.mark.parametrize("encoder_cache", [64, 0])
def test_repeated_media_served_from_encoder_caches(encoder_cache):
    from test_qwen3_omni_pipeline import TINY

    from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
    from sglang_omni_b200.config import PipelineRunner, compile_pipeline
    from sglang_omni_b200.models.qwen3_omni.config import Qwen3OmniPipelineConfig, text_stages

    cfg = Qwen3OmniPipelineConfig(model_path="random", stages=text_stages(
        overrides=TINY, device="cpu", max_batch=4, max_context=1024, encoder_cache=encoder_cache))
    rng = np.random.default_rng(3)
    audio = (rng.standard_normal(16000) * 0.1).astype(np.float32)
    image = rng.integers(0, 256, (64, 64, 3), dtype=np.uint8)

    async def main():
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            client = Client(coord)
            outs = []
            for i in range(3):
                req = GenerateRequest(prompt="describe", audios=[audio.copy()], images=[image.copy()], max_tokens=4,
                                      sampling=SamplingParams(temperature=0.0, ignore_eos=True),
                                      request_id=f"r{i}")
                outs.append((await client.completion(req)).token_ids)
            a, v = _engine_of(stages, "audio_encoder"), _engine_of(stages, "image_encoder")
            return outs, a.cache, v.cache

    outs, acache, vcache = asyncio.run(main())
    assert outs[0] == outs[1] == outs[2]
    if encoder_cache:
        assert (acache.hits, acache.misses) == (2, 1) and (vcache.hits, vcache.misses) == (2, 1)
    else:
        assert acache is None and vcache is None
