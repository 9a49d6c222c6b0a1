"""Page-granular prefix (radix) cache: the native tree on its own, and the paged
engine reusing cached prompt pages (outputs must equal a full recompute)."""
import numpy as np
import pytest
import torch

from sglang_omni_b200 import _runtime
from sglang_omni_b200.engines.ar import AREngine, ARRequest, KVPool
from sglang_omni_b200.models.decoder import DecoderLM
from sglang_omni_b200.sampling_params import SamplingParams

from test_ar_engine import check_greedy, tiny_cfg


def blocks(*vals):
    return np.concatenate([np.full(64, v, dtype=np.int32) for v in vals])


def test_tree_match_insert_evict():
    pc = _runtime.PrefixCache(64)
    nodes, pages = pc.match(0, blocks(1, 2, 3), 3)
    assert list(nodes) == [] and list(pages) == []
    assert list(pc.insert_release(0, blocks(1, 2, 3), [10, 11, 12], [])) == []
    assert pc.cached_pages() == 3 and pc.evictable_pages() == 3
    # longest run of full blocks; a different third block stops the match
    nodes, pages = pc.match(0, blocks(1, 2, 9), 3)
    assert list(pages) == [10, 11] and pc.evictable_pages() == 1
    # a second request inserting the same blocks hands its duplicate pages back
    dup = pc.insert_release(0, blocks(1, 2, 9), [10, 11, 20], list(nodes))
    assert list(dup) == [] and pc.cached_pages() == 4
    n2, p2 = pc.match(0, blocks(1, 2, 3), 3)
    dup = pc.insert_release(0, blocks(1, 2, 3), list(p2), list(n2))
    assert list(dup) == []
    assert list(pc.insert_release(0, blocks(1, 2, 3), [30, 31, 32], [])) == [30, 31, 32]
    # namespaces never share pages
    assert list(pc.match(7, blocks(1, 2, 3), 3)[1]) == []
    # locked paths are not evicted; the rest goes leaves first, least recent first
    held, hp = pc.match(0, blocks(1, 2, 9), 3)
    assert list(hp) == [10, 11, 20]
    assert sorted(pc.evict(10)) == [12]
    pc.release(list(held))
    with pytest.raises(RuntimeError):  # released more often than matched
        pc.release(list(held))
    out = pc.evict(10)
    assert out[0] == 20 and sorted(out) == [10, 11, 20]
    assert pc.cached_pages() == 0
    with pytest.raises(IndexError):  # evicted nodes are gone
        pc.release(list(held))


def shared_prefix_reqs(prefix, n, suffix_len, new, vocab, seed, tag):
    g = torch.Generator().manual_seed(seed)
    return [ARRequest(rid=f"{tag}{i}", prompt_ids=list(prefix) + torch.randint(0, vocab, (suffix_len + 3 * i,),
                                                                            generator=g).tolist(),
                      sampling=SamplingParams(temperature=0.0), max_new_tokens=new) for i in range(n)]


@pytest.mark.parametrize("overlap", [True, False])
def test_engine_reuses_prefix_cpu(overlap):
    cfg = tiny_cfg(False)
    model = DecoderLM(cfg).random_init_(seed=5, std=0.1)
    pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, 64, "cpu", cfg.dtype)
    eng = AREngine(model, pool, max_batch=4, max_prefill_tokens=96, max_context=512, use_graphs=False,
                   overlap=overlap, prefix_cache=True)
    prefix = torch.randint(0, cfg.vocab_size, (150,), generator=torch.Generator().manual_seed(9)).tolist()
    first = shared_prefix_reqs(prefix, 1, 20, 6, cfg.vocab_size, 1, "a")
    eng.generate(first)
    assert eng.num_prefix_hit_tokens == 0
    second = shared_prefix_reqs(prefix, 5, 10, 7, cfg.vocab_size, 2, "b")
    eng.generate(second)
    assert all(r.cached_tokens == 128 for r in second)  # two full pages of the shared 150-token prefix
    assert eng.num_prefix_hit_tokens == 5 * 128
    # the first request's own prompt + outputs come back whole (its last page is recomputed)
    again = [ARRequest(rid="c", prompt_ids=list(first[0].prompt_ids) + first[0].output_ids[:-1],
                       sampling=SamplingParams(temperature=0.0), max_new_tokens=3)]
    eng.generate(again)
    assert again[0].cached_tokens == 128
    check_greedy(model, first + second + again, "cpu", 1e-4)
    pc = eng.prefix_cache
    assert pool.free_pages + pc.cached_pages() == 63  # every page is free or owned by the tree
    assert pc.evictable_pages() == pc.cached_pages()  # nothing left locked


def test_engine_prefix_cache_evicts_under_pressure_cpu():
    cfg = tiny_cfg(True)
    model = DecoderLM(cfg).random_init_(seed=6, std=0.1)
    pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, 9, "cpu", cfg.dtype)  # 8 usable pages
    eng = AREngine(model, pool, max_batch=2, max_prefill_tokens=256, max_context=512, use_graphs=False,
                   prefix_cache=True)
    prefix = list(range(3, 3 + 130))
    reqs = []
    for wave in range(4):  # distinct prompts keep filling the tree; allocation must evict
        batch = shared_prefix_reqs(prefix if wave % 2 == 0 else [], 2, 70, 30, cfg.vocab_size, 10 + wave, f"w{wave}_")
        eng.generate(batch)
        reqs += batch
    assert all(len(r.output_ids) == 30 for r in reqs)
    assert eng.num_prefix_hit_tokens > 0
    check_greedy(model, reqs, "cpu", 1e-4)
    assert pool.free_pages + eng.prefix_cache.cached_pages() == 8


def test_engine_prefix_cache_skips_embedding_requests_cpu():
    cfg = tiny_cfg(False)
    model = DecoderLM(cfg).random_init_(seed=7, std=0.1)
    pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, 32, "cpu", cfg.dtype)
    eng = AREngine(model, pool, max_batch=2, max_prefill_tokens=256, max_context=512, use_graphs=False,
                   prefix_cache=True)
    ids = list(range(200))
    emb = torch.randn(200, cfg.hidden_size) * 0.1
    r1 = ARRequest(rid="e1", prompt_ids=ids, input_embeds=emb, sampling=SamplingParams(temperature=0.0),
                   max_new_tokens=2)
    r2 = ARRequest(rid="t1", prompt_ids=ids, sampling=SamplingParams(temperature=0.0), max_new_tokens=2,
                   extra={"prefix_key": "speaker-a"})
    r3 = ARRequest(rid="t2", prompt_ids=ids, sampling=SamplingParams(temperature=0.0), max_new_tokens=2)
    eng.generate([r1])
    eng.generate([r2])
    eng.generate([r3])
    assert r2.cached_tokens == 0 and r3.cached_tokens == 0  # other namespace / embeddings were never cached
    r4 = ARRequest(rid="t3", prompt_ids=ids, sampling=SamplingParams(temperature=0.0), max_new_tokens=2)
    eng.generate([r4])
    assert r4.cached_tokens == 192
    assert r4.output_ids == r3.output_ids
