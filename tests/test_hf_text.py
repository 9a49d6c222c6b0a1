"""Hugging Face causal LMs on this package's decoder: tiny random Llama (Llama-3 RoPE scaling),
Mistral, Qwen2 (q / k / v biases), Qwen3 (per-head q / k norm) and Qwen3-MoE checkpoints converted
to ``DecoderLM`` give transformers' logits, and a checkpoint directory served through the
registry's text pipeline generates transformers' greedy tokens."""
import asyncio
import math

import pytest
import torch

transformers = pytest.importorskip("transformers")

from sglang_omni_b200.engines.ar import KVPool  # noqa: E402
from sglang_omni_b200.models.decoder import ForwardBatch  # noqa: E402
from sglang_omni_b200.models.hf_text import decoder_config_from_hf, decoder_from_hf  # noqa: E402
from sglang_omni_b200.ops import prefill_tiles  # noqa: E402

BASE = dict(vocab_size=320, hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
            num_key_value_heads=2, max_position_embeddings=256, rms_norm_eps=1e-6, tie_word_embeddings=False)


def _hf(arch: str, seed: int = 0):
    extra = {}
    if arch == "llama":
        cfg = transformers.LlamaConfig(**BASE, rope_theta=5e5, rope_scaling={
            "rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
            "original_max_position_embeddings": 32})
    elif arch == "mistral":
        cfg = transformers.MistralConfig(**BASE, sliding_window=None, head_dim=24)
    elif arch == "qwen2":
        cfg = transformers.Qwen2Config(**{**BASE, "tie_word_embeddings": True})
    elif arch == "qwen3":
        cfg = transformers.Qwen3Config(**BASE, head_dim=32)
    else:
        cfg = transformers.Qwen3MoeConfig(**BASE, head_dim=16, num_experts=6, num_experts_per_tok=2,
                                          moe_intermediate_size=40, norm_topk_prob=True, mlp_only_layers=[1])
    cfg.architectures = [{"llama": "LlamaForCausalLM", "mistral": "MistralForCausalLM", "qwen2": "Qwen2ForCausalLM",
                          "qwen3": "Qwen3ForCausalLM", "qwen3moe": "Qwen3MoeForCausalLM"}[arch]]
    torch.manual_seed(seed)
    m = transformers.AutoModelForCausalLM.from_config(cfg, **extra).float().eval()
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if "norm" in n and n.endswith("weight"):
                p.copy_(1.0 + 0.1 * torch.randn(p.shape, generator=g))
            else:
                p.copy_(torch.randn(p.shape, generator=g) * (0.6 / math.sqrt(p.shape[-1])))
    return m


def _logits(model, tokens):
    cfg = model.cfg
    T = len(tokens)
    pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, (T + 63) // 64 + 2, "cpu", torch.float32)
    pages = pool.alloc((T + 63) // 64)
    t = torch.arange(T)
    slots = (torch.tensor(pages)[t // 64] * 64 + t % 64).to(torch.int32)
    req, tok0 = prefill_tiles([T], cfg.num_heads // cfg.num_kv_heads)
    fb = ForwardBatch(is_decode=False, positions=t.to(torch.int32), slot_mapping=slots,
                      kv_lens=torch.tensor([T], dtype=torch.int32), block_table=torch.tensor([pages], dtype=torch.int32),
                      input_ids=torch.tensor(tokens, dtype=torch.int32), cu_q=torch.tensor([0, T], dtype=torch.int32),
                      tile_req=torch.tensor(req, dtype=torch.int32), tile_tok0=torch.tensor(tok0, dtype=torch.int32))
    with torch.no_grad():
        return model.logits(model(fb, pool.kv)).float()


@pytest.mark.parametrize("arch", ["llama", "mistral", "qwen2", "qwen3", "qwen3moe"])
def test_converted_model_matches_transformers_logits(arch):
    hf = _hf(arch)
    ours = decoder_from_hf(hf, "cpu")
    tokens = torch.randint(0, BASE["vocab_size"], (70,), generator=torch.Generator().manual_seed(1)).tolist()
    with torch.no_grad():
        ref = hf(torch.tensor([tokens])).logits[0].float()
    got = _logits(ours, tokens)
    rel = float((got - ref).norm() / ref.norm())
    assert rel < 1e-4, (arch, rel)


def test_config_mapping_and_refusals():
    c = decoder_config_from_hf({"architectures": ["Qwen3MoeForCausalLM"], "vocab_size": 10, "hidden_size": 8,
                                "num_hidden_layers": 4, "num_attention_heads": 2, "num_experts": 4,
                                "num_experts_per_tok": 2, "moe_intermediate_size": 4, "decoder_sparse_step": 2,
                                "mlp_only_layers": [0], "rope_theta": 1e6})
    assert c.qk_norm and c.num_kv_heads == 2 and c.head_dim == 4
    assert [c.is_moe_layer(i) for i in range(4)] == [False, True, False, True]
    with pytest.raises(NotImplementedError, match="sliding-window"):
        decoder_config_from_hf({"architectures": ["MistralForCausalLM"], "vocab_size": 10, "hidden_size": 8,
                                "num_hidden_layers": 1, "num_attention_heads": 2, "sliding_window": 16,
                                "max_position_embeddings": 4096})
    with pytest.raises(ValueError, match="not one of"):
        decoder_config_from_hf({"architectures": ["GPT2LMHeadModel"], "vocab_size": 10, "hidden_size": 8,
                                "num_hidden_layers": 1, "num_attention_heads": 2})
    with pytest.raises(NotImplementedError, match="yarn"):
        decoder_config_from_hf({"architectures": ["Qwen2ForCausalLM"], "vocab_size": 10, "hidden_size": 8,
                                "num_hidden_layers": 1, "num_attention_heads": 2,
                                "rope_scaling": {"rope_type": "yarn", "factor": 4.0}})


def test_checkpoint_dir_served_through_registry(tmp_path):
    from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
    from sglang_omni_b200.config import ConfigManager, PipelineRunner, compile_pipeline

    hf = _hf("qwen3", seed=3)
    hf.generation_config.eos_token_id = None
    hf.save_pretrained(tmp_path, safe_serialization=True)
    cfg = ConfigManager.from_model_path(str(tmp_path))
    assert type(cfg).__name__ == "HFTextPipelineConfig"
    cfg = ConfigManager.merge_config(cfg, ConfigManager.parse_extra_args(
        ["--stages.1.executor.args.device", "cpu", "--stages.1.executor.args.max_context", "256",
         "--stages.1.executor.args.max_batch", "4", "--stages.1.executor.args.use_graphs", "false"]))
    prompt = torch.randint(0, 300, (12,), generator=torch.Generator().manual_seed(4)).tolist()
    with torch.no_grad():
        ref = hf.generate(torch.tensor([prompt]), max_new_tokens=8, do_sample=False, eos_token_id=None,
                          pad_token_id=0)[0, len(prompt):].tolist()

    async def run():
        coord, stages = compile_pipeline(cfg)
        async with PipelineRunner(coord, stages):
            client = Client(coord)
            req = GenerateRequest(prompt_token_ids=prompt, max_tokens=8,
                                  sampling=SamplingParams(temperature=0.0, ignore_eos=True))
            return await client.completion(req)

    res = asyncio.run(run())
    assert res.token_ids == ref


def test_create_ar_engine_takes_a_transformers_model():
    """The reference's factory signature: create_ar_engine(model=<HF causal LM>, tokenizer, max_seq_len,
    device) -> an engine whose greedy output equals transformers' generate."""
    from sglang_omni_b200.engines.ar import ARRequest
    from sglang_omni_b200.engines.omni.factory import create_ar_engine
    from sglang_omni_b200.sampling_params import SamplingParams

    hf = _hf("llama", seed=5)
    engine = create_ar_engine(hf, tokenizer=None, max_seq_len=128, device="cpu", max_batch=2, use_graphs=False)
    prompt = torch.randint(0, 300, (9,), generator=torch.Generator().manual_seed(6)).tolist()
    with torch.no_grad():
        ref = hf.generate(torch.tensor([prompt]), max_new_tokens=6, do_sample=False, eos_token_id=None,
                          pad_token_id=0)[0, len(prompt):].tolist()

    async def run():
        try:
            return await engine.generate("r0", ARRequest("r0", prompt, SamplingParams(temperature=0.0),
                                                         max_new_tokens=6))
        finally:
            engine.stop()

    assert asyncio.run(run()).output_ids == ref


@pytest.mark.gpu
def test_converted_llama_on_gpu_kernels_matches_transformers():
    """A converted Llama (Llama-3 RoPE scaling, GQA 4/2 x 64) on the sm_100a kernels in bf16 against
    transformers' fp32 logits on the CPU."""
    cfg = transformers.LlamaConfig(**{**BASE, "hidden_size": 256, "intermediate_size": 512}, rope_theta=5e5,
                                   rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                                 "high_freq_factor": 4.0, "original_max_position_embeddings": 32})
    cfg.architectures = ["LlamaForCausalLM"]
    torch.manual_seed(0)
    hf = transformers.AutoModelForCausalLM.from_config(cfg).float().eval()
    ours = decoder_from_hf(hf, "cuda")
    assert ours.cfg.dtype == torch.bfloat16 and ours.cfg.head_dim == 64
    tokens = torch.randint(0, BASE["vocab_size"], (150,), generator=torch.Generator().manual_seed(2)).tolist()
    with torch.no_grad():
        ref = hf(torch.tensor([tokens])).logits[0].float()
    c = ours.cfg
    T = len(tokens)
    pool = KVPool(c.num_layers, c.num_kv_heads, c.head_dim, (T + 63) // 64 + 2, "cuda", torch.bfloat16)
    pages = pool.alloc((T + 63) // 64)
    t = torch.arange(T)
    slots = (torch.tensor(pages)[t // 64] * 64 + t % 64).to(torch.int32)
    req, tok0 = prefill_tiles([T], c.num_heads // c.num_kv_heads)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device="cuda")  # noqa: E731
    fb = ForwardBatch(is_decode=False, positions=t.to(torch.int32).cuda(), slot_mapping=slots.cuda(),
                      kv_lens=i32([T]), block_table=i32([pages]), input_ids=i32(tokens), cu_q=i32([0, T]),
                      tile_req=i32(req), tile_tok0=i32(tok0))
    ours.ensure_workspaces(T, 1, 256)
    with torch.no_grad():
        got = ours.logits(ours(fb, pool.kv)).float().cpu()
    rel = float((got - ref).norm() / ref.norm())
    assert rel < 0.03, rel
