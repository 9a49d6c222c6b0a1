"""Paged AR engine (chunked prefill, overlap, retraction, CUDA-graph decode) vs teacher-forced full prefill."""
import pytest
import torch

from sglang_omni_b200.engines.ar import AREngine, ARRequest, KVPool
from sglang_omni_b200.models.decoder import DecoderConfig, DecoderLM, ForwardBatch
from sglang_omni_b200.ops import prefill_tile_rows, prefill_tiles
from sglang_omni_b200.sampling_params import SamplingParams


def tiny_cfg(moe=True, dtype=torch.float32, **kw):
    c = DecoderConfig(vocab_size=512, hidden_size=128, num_layers=2, num_heads=8, num_kv_heads=2, head_dim=64,
                      intermediate_size=256, num_experts=8 if moe else 0, topk=2 if moe else 0,
                      moe_intermediate_size=64, rope_theta=10000.0, mrope_section=[12, 10, 10] if moe else None,
                      qk_norm=True, max_position=4096, dtype=dtype)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def full_logits(model, tokens, device):
    """Teacher-forced logits of every position (fresh cache, one prefill)."""
    cfg = model.cfg
    T = len(tokens)
    pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, (T + 63) // 64 + 2, device, cfg.dtype)
    pages = pool.alloc((T + 63) // 64)
    t = torch.arange(T)
    slots = (torch.tensor(pages)[t // 64] * 64 + t % 64).to(torch.int32)
    G = cfg.num_heads // cfg.num_kv_heads
    rows = prefill_tile_rows(cfg.head_dim, G) if torch.device(device).type == "cuda" else 64
    req, tok0 = prefill_tiles([T], G, rows)
    pos = torch.arange(T, dtype=torch.int32)
    fb = ForwardBatch(is_decode=False, positions=torch.stack([pos] * 3).to(device), slot_mapping=slots.to(device),
                      kv_lens=torch.tensor([T], dtype=torch.int32, device=device),
                      block_table=torch.tensor([pages], dtype=torch.int32, device=device),
                      input_ids=torch.tensor(tokens, dtype=torch.int32, device=device),
                      cu_q=torch.tensor([0, T], dtype=torch.int32, device=device),
                      tile_req=torch.tensor(req, dtype=torch.int32, device=device),
                      tile_tok0=torch.tensor(tok0, dtype=torch.int32, device=device), tile_rows=rows)
    h = model(fb, pool.kv)
    return model.logits(h).float().cpu()


def check_greedy(model, reqs, device, tol):
    for r in reqs:
        seq = list(r.prompt_ids) + r.output_ids
        lg = full_logits(model, seq, device)
        for i, tok in enumerate(r.output_ids):
            row = lg[len(r.prompt_ids) - 1 + i]
            assert row[tok] >= row.max() - tol, (r.rid, i, float(row.max() - row[tok]))


def make_reqs(n, plen_fn, new, vocab, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for i in range(n):
        L = plen_fn(i)
        ids = torch.randint(0, vocab, (L,), generator=g).tolist()
        out.append(ARRequest(rid=f"r{i}", prompt_ids=ids, sampling=SamplingParams(temperature=0.0),
                             max_new_tokens=new))
    return out


@pytest.mark.parametrize("moe", [True, False])
@pytest.mark.parametrize("overlap", [True, False])
def test_engine_cpu_matches_full_recompute(moe, overlap):
    torch.manual_seed(0)
    cfg = tiny_cfg(moe)
    model = DecoderLM(cfg).random_init_(seed=1, std=0.1)
    pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, 64, "cpu", cfg.dtype)
    eng = AREngine(model, pool, max_batch=4, max_prefill_tokens=48, max_context=512, use_graphs=False,
                   overlap=overlap)
    reqs = make_reqs(6, lambda i: 5 + 17 * i, 9, cfg.vocab_size)
    eng.generate(reqs)
    assert all(len(r.output_ids) == 9 for r in reqs)
    assert pool.free_pages == 63  # everything returned
    check_greedy(model, reqs, "cpu", 1e-4)


def test_engine_retraction_cpu():
    cfg = tiny_cfg(False)
    model = DecoderLM(cfg).random_init_(seed=2, std=0.1)
    pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, 6, "cpu", cfg.dtype)  # 5 usable pages
    eng = AREngine(model, pool, max_batch=3, max_prefill_tokens=256, max_context=512, use_graphs=False)
    reqs = make_reqs(3, lambda i: 60, 40, cfg.vocab_size, seed=3)
    eng.generate(reqs)
    assert eng.num_retractions >= 1
    assert all(len(r.output_ids) == 40 for r in reqs)
    check_greedy(model, reqs, "cpu", 1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("graphs", [True, False])
def test_engine_gpu_graphs(graphs):
    cfg = tiny_cfg(True, dtype=torch.bfloat16, num_experts=16, topk=4, hidden_size=256, num_heads=16,
                   num_kv_heads=2, head_dim=128, moe_intermediate_size=128, mrope_section=[24, 20, 20],
                   vocab_size=1024)
    model = DecoderLM(cfg, device="cuda").random_init_(seed=4, std=0.05)
    pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, 256, "cuda", cfg.dtype)
    eng = AREngine(model, pool, max_batch=8, max_prefill_tokens=200, max_context=1024, use_graphs=graphs)
    reqs = make_reqs(11, lambda i: 3 + 31 * i, 20, cfg.vocab_size, seed=5)
    eng.generate(reqs)
    assert all(len(r.output_ids) == 20 for r in reqs)
    check_greedy(model, reqs, "cuda", 0.15)
