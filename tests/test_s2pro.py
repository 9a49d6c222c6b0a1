"""FishAudio S2-Pro: prompt layout, VQ input embedding, DAC codec vs an fp32
oracle, batched dual-AR generation, and the 3-stage TTS pipeline end to end."""
import asyncio

import numpy as np
import pytest
import torch

from sglang_omni_b200.models.fishaudio_s2_pro.codec import (DACConfig, DACDecoder, DACEncoder, dac_decode_reference,
                                                            random_dac_state_dict)
from sglang_omni_b200.models.fishaudio_s2_pro.generator import DualARGenerator
from sglang_omni_b200.models.fishaudio_s2_pro.hf_config import S2ProConfig, fast_config, slow_config
from sglang_omni_b200.models.fishaudio_s2_pro.model import S2ProDualAR
from sglang_omni_b200.models.fishaudio_s2_pro.tokenizer import (FishFallbackTokenizer, Reference,
                                                                S2ProPromptBuilder)
from sglang_omni_b200.ops.embedding import vq_embed, vq_embed_ref

DAC_TINY = dict(latent_dim=64, decoder_dim=128, tf_layers=2, tf_heads=1, tf_head_dim=64, tf_inter=128,
                tf_window=8, encoder_dim=8, encoder_transformer_layers=(0, 0, 0, 1), n_codebooks=3,
                codebook_size=32, semantic_codebook_size=64)
TINY = {
    "slow": {"vocab_size": 512, "hidden_size": 64, "num_layers": 2, "num_heads": 4, "num_kv_heads": 2,
             "head_dim": 64, "intermediate_size": 128},
    "fast": {"hidden_size": 64, "num_layers": 2, "num_heads": 4, "num_kv_heads": 2, "head_dim": 64,
             "intermediate_size": 128},
    "s2pro": {"codebook_size": 64, "num_codebooks": 4},
    "dac": DAC_TINY,
}


def tiny_model(device="cpu", dtype=torch.float32, seed=3):
    tok = FishFallbackTokenizer(512, 64)
    cfg = S2ProConfig(slow=slow_config(**TINY["slow"], dtype=dtype), fast=fast_config(**TINY["fast"], dtype=dtype),
                      num_codebooks=4, codebook_size=64, semantic_begin_id=tok.semantic_begin_id,
                      im_end_id=tok.convert_tokens_to_ids("<|im_end|>"))
    cfg.fast.vocab_size = 64
    return S2ProDualAR(cfg, device).random_init_(seed=seed, std=0.2), tok


def test_prompt_layout():
    tok = FishFallbackTokenizer()
    b = S2ProPromptBuilder(tok, 10)
    codes = torch.randint(0, 1024, (10, 7))
    p = b.build("hello", [Reference(text="ref words", vq_codes=codes)])
    assert sum(p.vq_mask) == 7 and p.vq_codes.shape == (7, 10)
    first = p.vq_mask.index(True)
    assert p.ids[first: first + 7] == [tok.semantic_begin_id + int(c) for c in codes[0]]
    assert torch.equal(p.vq_codes, codes.t().to(torch.int32))
    text = tok.decode(p.ids, skip_special_tokens=False)
    assert text.startswith("<|im_start|>system\nconvert the provided text to speech reference")
    assert "<|speaker:0|>ref words\n\nSpeech:\n<|semantic:" in text
    assert text.endswith("<|im_start|>user\n<|speaker:0|>hello<|im_end|>\n<|im_start|>assistant\n<|voice|>")
    rows = p.code_rows()
    assert rows[first].item() == 0 and rows[first + 6].item() == 6 and rows[0].item() == -1
    q = b.build("plain")
    assert sum(q.vq_mask) == 0 and tok.decode(q.ids, False).startswith("<|im_start|>user\n")


def test_vq_embed_ref_definition():
    torch.manual_seed(0)
    E = torch.randn(300, 16)
    CB = torch.randn(3 * 10, 16)
    codes = torch.randint(0, 10, (5, 3), dtype=torch.int32)
    ids = torch.tensor([1, 250, 7, 251, 3], dtype=torch.int32)
    rows = torch.tensor([-1, 0, -1, 3, -1], dtype=torch.int32)
    out = vq_embed(E, CB, codes, 10, 0.5, 250, 259, ids=ids, code_row=rows)
    assert torch.equal(out[0], E[1])
    want = (E[250] + CB[codes[0, 0]] + CB[10 + codes[0, 1]] + CB[20 + codes[0, 2]]) * 0.5
    torch.testing.assert_close(out[1], want)
    slot_tok = torch.tensor([0, 250, 5], dtype=torch.int32)
    out2 = vq_embed(E, CB, codes, 10, 0.5, 250, 259, slot=torch.tensor([1, 2], dtype=torch.int32),
                    slot_tokens=slot_tok)
    torch.testing.assert_close(out2[0], (E[250] + CB[codes[1, 0]] + CB[10 + codes[1, 1]] + CB[20 + codes[1, 2]]) * .5)
    assert torch.equal(out2[1], E[5])


def test_dac_decoder_matches_reference_cpu():
    cfg = DACConfig(**DAC_TINY, dtype=torch.float32)
    sd = random_dac_state_dict(cfg, seed=1, std=0.1)
    codes = torch.stack([torch.randint(0, 64, (2, 11))] + [torch.randint(0, 40, (2, 11)) for _ in range(3)], 1)
    ref = dac_decode_reference(sd, codes, cfg)
    out = DACDecoder(cfg).load_state_dict_dac(sd).decode(codes)
    assert out.shape == (2, 11 * cfg.hop)
    assert float((out - ref).norm() / ref.norm()) < 1e-4


def test_dac_encoder_codes_in_range():
    cfg = DACConfig(**DAC_TINY, dtype=torch.float32)
    enc = DACEncoder(random_dac_state_dict(cfg, seed=2, std=0.1), cfg)
    c = enc.encode(torch.randn(1, 3 * cfg.hop + 100) * 0.1)
    assert c.shape == (1, 4, 4)
    assert int(c[:, 0].max()) < 64 and int(c[:, 1:].max()) < 32


def _run(gen, tok, prompts, frames, greedy=True):
    out = {}
    streams = []
    for i, p in enumerate(prompts):
        streams.append(gen.add_stream(f"r{i}", p.ids, p.code_rows(), p.vq_codes, max_new_tokens=frames,
                                      temperature=0.0 if greedy else 0.8))
    codes = gen.prefill(streams)
    for s, c in zip(streams, codes.tolist()):
        out[s.rid] = [c]
    for _ in range(frames - 1):
        codes = gen.step(streams)
        for s, c in zip(streams, codes.tolist()):
            out[s.rid].append(c)
    for s in streams:
        gen.remove(s.rid)
    return out


def test_generator_batched_matches_single_cpu():
    model, tok = tiny_model()
    b = S2ProPromptBuilder(tok, 4)
    prompts = [b.build("first one"), b.build("second, longer text", [Reference("r", torch.randint(0, 30, (4, 5)))]),
               b.build("x")]
    gen = DualARGenerator(model, max_streams=4, max_context=256, use_graphs=False)
    batched = _run(gen, tok, prompts, 4)
    for i, p in enumerate(prompts):
        single = _run(gen, tok, [p], 4)
        assert single["r0"] == batched[f"r{i}"], i
    for frames in batched.values():
        for c in frames:
            assert c[0] == tok.convert_tokens_to_ids("<|im_end|>") or \
                tok.semantic_begin_id <= c[0] < tok.semantic_begin_id + 64
            assert all(0 <= x < 64 for x in c[1:])


def _pipeline_run(device, stream: bool, n: int = 2):
    from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
    from sglang_omni_b200.config import PipelineRunner, compile_pipeline
    from sglang_omni_b200.models.fishaudio_s2_pro.config import S2ProPipelineConfig, s2pro_stages

    cfg = S2ProPipelineConfig(model_path="random", stages=s2pro_stages(overrides=TINY, device=device, max_new_tokens=6,
                                                                        max_streams=4, max_context=512,
                                                                        stream_stride=2, stream_followup_stride=2))

    async def main():
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            client = Client(coord)

            async def one(i):
                req = GenerateRequest(prompt=f"say number {i}", sampling=SamplingParams(temperature=0.0),
                                      output_modalities=["audio"], task="tts", stream=stream,
                                      metadata={"references": [{"text": "ref", "vq_codes": [[1, 2, 3]] * 4}]})
                chunks, final = [], None
                async for ch in client.generate(req):
                    if ch.finish_reason is not None:
                        final = ch
                    elif ch.modality == "audio" and ch.audio_data is not None:
                        chunks.append(np.asarray(ch.audio_data))
                return chunks, final

            return await asyncio.gather(*[one(i) for i in range(n)])

    return asyncio.run(main())


def test_s2pro_pipeline_cpu_end_to_end():
    for stream in (False, True):
        res = _pipeline_run("cpu", stream)
        for chunks, final in res:
            assert final is not None and final.audio_data is not None
            n = np.asarray(final.audio_data).size
            assert n > 0 and n % 2048 == 0 and n <= 6 * 2048
            assert final.sample_rate == 44100
            if stream:
                assert chunks and sum(c.size for c in chunks) == n
                # the stateful stream decoder's chunks add up to the vocoder stage's full decode
                np.testing.assert_allclose(np.concatenate(chunks).reshape(-1),
                                           np.asarray(final.audio_data, dtype=np.float32).reshape(-1),
                                           atol=1e-4, rtol=1e-3)


@pytest.mark.gpu
def test_vq_embed_gpu_matches_ref():
    torch.manual_seed(0)
    E = torch.randn(1000, 256).bfloat16().cuda()
    CB = torch.randn(10 * 64, 256).bfloat16().cuda()
    codes = torch.randint(0, 64, (40, 10), dtype=torch.int32).cuda()
    ids = torch.randint(0, 1000, (40,), dtype=torch.int32).cuda()
    rows = torch.where(torch.rand(40, device="cuda") < 0.5, torch.arange(40, device="cuda"), -1).to(torch.int32)
    out = vq_embed(E, CB, codes, 64, 11 ** -0.5, 900, 999, ids=ids, code_row=rows)
    ref = vq_embed_ref(E.cpu(), CB.cpu(), codes.cpu(), 64, 11 ** -0.5, 900, 999, ids=ids.cpu(), code_row=rows.cpu())
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=2e-2, rtol=1e-2)
    slot = torch.tensor([3, 1, 0], dtype=torch.int32).cuda()
    st = torch.tensor([950, 10, 990, 920], dtype=torch.int32).cuda()
    out2 = vq_embed(E, CB, codes, 64, 0.3, 900, 999, slot=slot, slot_tokens=st)
    ref2 = vq_embed_ref(E.cpu(), CB.cpu(), codes.cpu(), 64, 0.3, 900, 999, slot=slot.cpu(), slot_tokens=st.cpu())
    torch.testing.assert_close(out2.cpu().float(), ref2.float(), atol=2e-2, rtol=1e-2)


@pytest.mark.gpu
def test_dac_decoder_gpu_matches_reference():
    cfg = DACConfig(**DAC_TINY)
    sd = random_dac_state_dict(cfg, seed=4, std=0.05)
    codes = torch.stack([torch.randint(0, 64, (2, 9))] + [torch.randint(0, 32, (2, 9)) for _ in range(3)], 1)
    ref = dac_decode_reference(sd, codes, DACConfig(**DAC_TINY, dtype=torch.float32))
    out = DACDecoder(cfg, "cuda").load_state_dict_dac(sd).decode(codes.cuda()).cpu()
    assert float((out - ref).norm() / ref.norm()) < 0.05


@pytest.mark.gpu
def test_generator_gpu_graphs_match_eager():
    model, tok = tiny_model("cuda", torch.bfloat16, seed=5)
    b = S2ProPromptBuilder(tok, 4)
    prompts = [b.build("alpha"), b.build("beta gamma", [Reference("r", torch.randint(0, 30, (4, 6)))])]
    eager = _run(DualARGenerator(model, max_streams=4, max_context=256, use_graphs=False), tok, prompts, 5)
    graphs = _run(DualARGenerator(model, max_streams=4, max_context=256, use_graphs=True), tok, prompts, 5)
    assert eager == graphs


@pytest.mark.gpu
def test_s2pro_pipeline_gpu_end_to_end():
    res = _pipeline_run("cuda:0", True, n=3)
    for chunks, final in res:
        assert final is not None and np.asarray(final.audio_data).size % 2048 == 0
        assert chunks
