"""Talker + code predictor runtime: batched lock-step streams must produce the
same codes as each stream alone (greedy), prefill layout and EOS handling."""
import pytest
import torch

from sglang_omni_b200.models.decoder import DecoderConfig
from sglang_omni_b200.models.qwen3_omni.talker import (Qwen3OmniTalker, SpeechGenerator, TalkerSpecialTokens,
                                                        build_talker_prefill)


def tiny(dtype=torch.float32, device="cpu"):
    sp = TalkerSpecialTokens(codec_eos=250, codec_nothink=251, codec_think_bos=252, codec_think_eos=253,
                             codec_pad=254, codec_bos=255, speakers={"a": 240}, default_speaker="a",
                             tts_pad=90, tts_bos=91, tts_eos=92, im_start=93, im_end=94, system=95, user=96,
                             assistant=97, newline=98, num_code_groups=4)
    tc = DecoderConfig(vocab_size=256, hidden_size=64, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64,
                       intermediate_size=96, num_experts=8, topk=2, moe_intermediate_size=32,
                       shared_expert_intermediate_size=64, rope_theta=1e4, mrope_section=[12, 10, 10], dtype=dtype)
    cc = DecoderConfig(vocab_size=64, hidden_size=64, num_layers=2, num_heads=4, num_kv_heads=2, head_dim=64,
                       intermediate_size=96, rope_theta=1e4, max_position=64, dtype=dtype)
    t = Qwen3OmniTalker(tc, cc, thinker_hidden=48, special=sp, device=device).random_init_(seed=1, std=0.2)
    emb = (torch.randn(100, 48, generator=torch.Generator().manual_seed(2)) * 0.5).to(dtype).to(device)
    return t, emb


def _gen(t, emb, rids, frames, device="cpu"):
    g = SpeechGenerator(t, emb, max_streams=4, max_context=256, max_trailing=32, use_graphs=device != "cpu",
                        talker_sampling=(0.0, 0, 1.0, 1.0), cp_sampling=(0.0, 0, 1.0))
    prompts = {"a": [93, 96, 10, 11, 12, 94, 93, 97], "b": [93, 96, 20, 21, 94, 93, 97]}
    out = {}
    streams = []
    for r in rids:
        pre, trail, pad_e, eos_e = build_talker_prefill(t, emb, prompts[r], [30, 31, 32] if r == "a" else [40])
        streams.append(g.add_stream(r, pre, trail, pad_e, eos_e, thinker_done=True))
    codes0 = g.prefill(streams)
    for s, c in zip(streams, codes0):
        out[s.rid] = [c.tolist()]
    for _ in range(frames):
        ready = g.ready_streams()
        codes = g.step(ready)
        for s, c in zip(ready, codes):
            out[s.rid].append(c.tolist())
    return out


def test_batched_streams_match_single_cpu():
    t, emb = tiny()
    both = _gen(t, emb, ["a", "b"], 5)
    alone_a = _gen(t, emb, ["a"], 5)
    alone_b = _gen(t, emb, ["b"], 5)
    assert both["a"] == alone_a["a"]
    assert both["b"] == alone_b["b"]
    assert len(both["a"]) == 6 and len(both["a"][0]) == 4


def test_prefill_layout():
    t, emb = tiny()
    pre, trail, pad_e, eos_e = build_talker_prefill(t, emb, [93, 95, 1, 94, 93, 96, 10, 11, 94, 93, 97], [30, 31])
    # system segment skipped, user segment 5 tokens, assistant part 9 rows
    assert pre.shape[0] == 5 + 9
    assert trail.shape[0] == 1  # response tokens after the first


@pytest.mark.gpu
def test_batched_streams_match_single_gpu_graphs():
    t, emb = tiny(torch.bfloat16, "cuda")
    both = _gen(t, emb, ["a", "b"], 6, device="cuda")
    alone_a = _gen(t, emb, ["a"], 6, device="cuda")
    assert len(both["a"]) == 7
    # greedy + per-row independent kernels: batching must not change a stream's codes
    assert both["a"] == alone_a["a"]
