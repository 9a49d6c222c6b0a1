"""Tensor parallelism over peer memory on 2 GPUs (one process per GPU): the
sharded decoder (local heads, local experts / MLP slices, fused owner-scatter
epilogues + reduce/RMSNorm/all-gather kernel) must match the unsharded model of
the same weights, for a prefill and for engine decode steps (eager and CUDA
graphs).  Host-side pieces (head split, weight slices) also run on the CPU."""
import os
import socket

import pytest
import torch

from sglang_omni_b200.models.decoder import DecoderConfig, DecoderLM


def _cfg(moe: bool, **kw):
    c = DecoderConfig(vocab_size=512, hidden_size=256, num_layers=3, num_heads=8, num_kv_heads=2, head_dim=64,
                      intermediate_size=512, num_experts=16 if moe else 0, topk=4 if moe else 0,
                      moe_intermediate_size=128, shared_expert_intermediate_size=128 if moe else 0,
                      rope_theta=10000.0, mrope_section=[12, 10, 10], qk_norm=True, max_position=4096,
                      dtype=torch.bfloat16)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def test_head_split_gqa_groups():
    from sglang_omni_b200.parallel.tp import head_split

    for world in (1, 2, 4, 8):
        qs, kvs = [], []
        for r in range(world):
            q, kv = head_split(32, 4, r, world)
            qs += list(q)
            kvs.append(list(kv))
            assert all(h // 8 in kv for h in q)
        assert qs == list(range(32))
    assert head_split(32, 4, 5, 8)[1] == range(2, 3)


class _FakeTP:
    def __init__(self, rank, world):
        self.rank, self.world = rank, world


def test_shards_reassemble_cpu():
    """Concatenating every rank's slices gives back the unsharded tensors."""
    from sglang_omni_b200.parallel.tp import head_split
    from sglang_omni_b200.parallel.vocab import vocab_slice

    cfg = _cfg(True, dtype=torch.float32)
    full = DecoderLM(cfg).random_init_(seed=3)
    world = 2
    parts = [DecoderLM(cfg, tp=_FakeTP(r, world)).random_init_(seed=3) for r in range(world)]
    L0 = full.layers[1]
    D, qs, kvs = cfg.head_dim, cfg.q_size, cfg.kv_size
    for r, m in enumerate(parts):
        q, kv = head_split(cfg.num_heads, cfg.num_kv_heads, r, world)
        P = m.layers[1]
        assert torch.equal(P.qkv[:len(q) * D], L0.qkv[q.start * D:q.stop * D])
        assert torch.equal(P.qkv[len(q) * D:len(q) * D + len(kv) * D], L0.qkv[qs + kv.start * D:qs + kv.stop * D])
        assert torch.equal(P.o, L0.o[:, q.start * D:q.stop * D])
        El = cfg.num_experts // world
        assert torch.equal(P.w13, L0.w13[r * El:(r + 1) * El])
        Is = cfg.shared_expert_intermediate_size // world
        assert torch.equal(P.s13[:Is], L0.s13[r * Is:(r + 1) * Is])
        assert torch.equal(P.s2, L0.s2[:, r * Is:(r + 1) * Is])
        assert torch.equal(P.router, L0.router) and torch.equal(m.embed, full.embed)
        assert m.cfg.num_heads == cfg.num_heads // world and m.cfg.num_kv_heads == 1
        # vocab-parallel LM head: this rank's vocabulary rows, zero padded to the slice width
        v0, vl, width = vocab_slice(cfg.vocab_size, r, world)
        assert m.lm_head.shape[0] == width
        assert torch.equal(m.lm_head[:vl], full.lm_head[v0:v0 + vl]) and not m.lm_head[vl:].any()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ds_logits(model, tokens, device, deepstack):
    """Teacher-forced logits of one prefill with deep-stack rows added after layers 0 .. n-1."""
    from sglang_omni_b200.engines.ar import KVPool
    from sglang_omni_b200.models.decoder import ForwardBatch
    from sglang_omni_b200.ops import prefill_tile_rows, prefill_tiles

    cfg = model.cfg
    T = len(tokens)
    pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, (T + 63) // 64 + 2, device, cfg.dtype)
    pages = pool.alloc((T + 63) // 64)
    t = torch.arange(T)
    slots = (torch.tensor(pages)[t // 64] * 64 + t % 64).to(torch.int32)
    G = cfg.num_heads // cfg.num_kv_heads
    rows = prefill_tile_rows(cfg.head_dim, G)
    req, tok0 = prefill_tiles([T], G, rows)
    pos = torch.arange(T, dtype=torch.int32)
    d = lambda x: x.to(device)  # noqa: E731
    fb = ForwardBatch(is_decode=False, positions=d(torch.stack([pos] * 3)), slot_mapping=d(slots),
                      kv_lens=d(torch.tensor([T], dtype=torch.int32)), block_table=d(torch.tensor([pages],
                                                                                                   dtype=torch.int32)),
                      input_ids=d(torch.tensor(tokens, dtype=torch.int32)), cu_q=d(torch.tensor([0, T],
                                                                                             dtype=torch.int32)),
                      tile_req=d(torch.tensor(req, dtype=torch.int32)), tile_tok0=d(torch.tensor(tok0,
                                                                                              dtype=torch.int32)),
                      tile_rows=rows, deepstack=list(deepstack))
    return model.logits(model(fb, pool.kv)).float().cpu()


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=60))
        from sglang_omni_b200.engines.ar import AREngine, ARRequest, KVPool
        from sglang_omni_b200.ops._ext import check_status
        from sglang_omni_b200.parallel import TPGroup
        from sglang_omni_b200.sampling_params import SamplingParams
        from test_ar_engine import full_logits

        errs = {}
        for moe in (True, False):
            cfg = _cfg(moe)
            ref = DecoderLM(cfg, device=dev).random_init_(seed=11, std=0.05)
            tp = TPGroup(cfg.hidden_size, 512, dev)
            m = DecoderLM(cfg, device=dev, tp=tp).random_init_(seed=11, std=0.05)
            toks = torch.randint(0, cfg.vocab_size, (150,), generator=torch.Generator().manual_seed(5)).tolist()
            a = full_logits(ref, toks, dev)
            b = full_logits(m, toks, dev)
            torch.cuda.synchronize()
            check_status(dev)
            errs[f"prefill_moe{moe}"] = float((a - b).norm() / a.norm())
            # deep-stack rows injected into the first two layers' outputs (vision positions 10..41)
            gds = torch.Generator(device=dev).manual_seed(9)
            pos = torch.arange(10, 42, device=dev)
            ds = [(pos, torch.randn(32, cfg.hidden_size, device=dev, generator=gds).bfloat16()) for _ in range(2)]
            a = _ds_logits(ref, toks, dev, ds)
            b = _ds_logits(m, toks, dev, ds)
            errs[f"prefill_deepstack_moe{moe}"] = float((a - b).norm() / a.norm())
            # engine: greedy decode, graphs on / off, identical requests on both ranks
            for graphs in (False, True):
                pool = KVPool(m.cfg.num_layers, m.cfg.num_kv_heads, m.cfg.head_dim, 128, dev, m.cfg.dtype)
                eng = AREngine(m, pool, max_batch=4, max_prefill_tokens=128, max_context=512, use_graphs=graphs)
                g = torch.Generator().manual_seed(7)
                reqs = [ARRequest(rid=f"r{i}", prompt_ids=torch.randint(0, cfg.vocab_size, (20 + 13 * i,),
                                                                       generator=g).tolist(),
                                  sampling=SamplingParams(temperature=0.0, ignore_eos=True), max_new_tokens=12)
                        for i in range(5)]
                eng.generate(reqs)
                torch.cuda.synchronize()
                check_status(dev)
                worst = 0.0
                for r in reqs:
                    lg = full_logits(ref, list(r.prompt_ids) + r.output_ids, dev)
                    for i, tok in enumerate(r.output_ids):
                        row = lg[len(r.prompt_ids) - 1 + i]
                        worst = max(worst, float(row.max() - row[tok]))
                errs[f"greedy_gap_moe{moe}_graphs{graphs}"] = worst
                # both ranks produced the same tokens
                mine = torch.tensor([t for r in reqs for t in r.output_ids], device=dev)
                other = mine.clone()
                dist.broadcast(other, 0)
                errs[f"rank_mismatch_moe{moe}_graphs{graphs}"] = float((mine != other).sum())
                # sampled decode through the vocab-parallel head: every rank draws the same tokens
                for r in reqs:
                    r.output_ids.clear()
                sreqs = [ARRequest(rid=f"s{i}", prompt_ids=list(r.prompt_ids),
                                   sampling=SamplingParams(temperature=0.8, top_k=20, seed=100 + i, ignore_eos=True),
                                   max_new_tokens=12) for i, r in enumerate(reqs)]
                eng.generate(sreqs)
                torch.cuda.synchronize()
                check_status(dev)
                mine = torch.tensor([t for r in sreqs for t in r.output_ids], device=dev)
                other = mine.clone()
                dist.broadcast(other, 0)
                errs[f"sampled_rank_mismatch_moe{moe}_graphs{graphs}"] = float((mine != other).sum())
                errs[f"vocab_inexact_moe{moe}_graphs{graphs}"] = float(m.vocab_sampler.inexact_rows)
                eng = pool = None
            m = None
            import gc

            gc.collect()
            torch.cuda.synchronize()
            tp.close()
        dist.destroy_process_group()
        q.put((rank, errs, None))
    except Exception:  # report instead of hanging the parent
        import traceback

        q.put((rank, None, traceback.format_exc()))


def _worker_tpep(rank, world, port, q):
    """Attention TP over both ranks combined with expert-parallel MoE over both ranks."""
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=60))
        from sglang_omni_b200.engines.ar import AREngine, ARRequest, KVPool
        from sglang_omni_b200.ops._ext import check_status
        from sglang_omni_b200.parallel import EPMoE, TPGroup
        from sglang_omni_b200.sampling_params import SamplingParams
        from test_ar_engine import full_logits

        errs = {}
        cfg = _cfg(True)
        ref = DecoderLM(cfg, device=dev).random_init_(seed=11, std=0.05)
        tp = TPGroup(cfg.hidden_size, 512, dev)
        ep = EPMoE(cfg.num_experts, cfg.topk, cfg.hidden_size, cfg.moe_intermediate_size, max_tokens=512,
                   device=dev)
        m = DecoderLM(cfg, device=dev, tp=tp, ep=ep).random_init_(seed=11, std=0.05)
        assert m.layers[1].w13.shape[0] == cfg.num_experts // world
        assert m.layers[1].s13.shape[0] == 2 * cfg.shared_expert_intermediate_size   # shared expert whole
        toks = torch.randint(0, cfg.vocab_size, (150,), generator=torch.Generator().manual_seed(5)).tolist()
        a = full_logits(ref, toks, dev)
        b = full_logits(m, toks, dev)
        torch.cuda.synchronize()
        check_status(dev)
        errs["prefill_tpep"] = float((a - b).norm() / a.norm())
        for graphs in (False, True):
            pool = KVPool(m.cfg.num_layers, m.cfg.num_kv_heads, m.cfg.head_dim, 128, dev, m.cfg.dtype)
            eng = AREngine(m, pool, max_batch=4, max_prefill_tokens=128, max_context=512, use_graphs=graphs)
            g = torch.Generator().manual_seed(7)
            reqs = [ARRequest(rid=f"r{i}", prompt_ids=torch.randint(0, cfg.vocab_size, (20 + 13 * i,),
                                                                   generator=g).tolist(),
                              sampling=SamplingParams(temperature=0.0, ignore_eos=True), max_new_tokens=10)
                    for i in range(5)]
            eng.generate(reqs)
            torch.cuda.synchronize()
            check_status(dev)
            worst = 0.0
            for r in reqs:
                lg = full_logits(ref, list(r.prompt_ids) + r.output_ids, dev)
                for i, tok in enumerate(r.output_ids):
                    row = lg[len(r.prompt_ids) - 1 + i]
                    worst = max(worst, float(row.max() - row[tok]))
            errs[f"greedy_gap_tpep_graphs{graphs}"] = worst
            mine = torch.tensor([t for r in reqs for t in r.output_ids], device=dev)
            other = mine.clone()
            dist.broadcast(other, 0)
            errs[f"rank_mismatch_tpep_graphs{graphs}"] = float((mine != other).sum())
            eng = pool = None
        m.close_parallel()
        dist.destroy_process_group()
        q.put((rank, errs, None))
    except Exception:  # report instead of hanging the parent
        import traceback

        q.put((rank, None, traceback.format_exc()))


def _run2(target):
    import sys

    import torch.multiprocessing as mp

    sys.path.insert(0, os.path.dirname(__file__))
    world = 2
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, qu)) for r in range(world)]
    for p in procs:
        p.start()
    res = [qu.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return res


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_ep_combined_matches_unsharded():
    for rank, errs, tb in _run2(_worker_tpep):
        assert tb is None, tb
        for k, v in errs.items():
            if k.startswith("prefill"):
                assert v < 0.03, (rank, k, v)
            elif k.startswith("greedy"):
                assert v < 0.2, (rank, k, v)
            else:
                assert v == 0, (rank, k, v)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_matches_unsharded():
    import sys

    import torch.multiprocessing as mp

    sys.path.insert(0, os.path.dirname(__file__))
    world = 2
    ctx = mp.get_context("spawn")
    qu = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, qu)) for r in range(world)]
    for p in procs:
        p.start()
    res = [qu.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, errs, tb in res:
        assert tb is None, tb
        for k, v in errs.items():
            if k.startswith("prefill"):
                assert v < 0.03, (rank, k, v)
            elif k.startswith("greedy"):
                assert v < 0.2, (rank, k, v)
            else:
                assert v == 0, (rank, k, v)


def test_qkv_bias_shards_through_the_loader_cpu():
    """Q / K / V biases (Qwen2-style layers, e.g. the Ming talker's LM) load into each TP rank as
    the rows of its heads, the same slices as the QKV weight."""
    from sglang_omni_b200.models.weight_loader import export_decoder_to_hf, load_decoder_from_hf
    from sglang_omni_b200.parallel.tp import head_split

    cfg = _cfg(False, dtype=torch.float32, attention_bias=True)
    full = DecoderLM(cfg).random_init_(seed=5)
    with torch.no_grad():
        for L in full.layers:
            L.qkv_bias.normal_(0.0, 0.1)
    sd = export_decoder_to_hf(full)
    world = 2
    D = cfg.head_dim
    for r in range(world):
        m = DecoderLM(cfg, tp=_FakeTP(r, world))
        load_decoder_from_hf(m, sd, "model.", "lm_head.weight")
        q, kv = head_split(cfg.num_heads, cfg.num_kv_heads, r, world)
        for L0, L in zip(full.layers, m.layers):
            b = L0.qkv_bias
            want = torch.cat([b[q.start * D:q.stop * D], b[cfg.q_size + kv.start * D:cfg.q_size + kv.stop * D],
                              b[cfg.q_size + cfg.kv_size + kv.start * D:cfg.q_size + cfg.kv_size + kv.stop * D]])
            assert torch.equal(L.qkv_bias, want)
            assert torch.equal(L.qkv, m.shard("qkv", L0.qkv))
