"""Thinker stages served by a rank group on 2 / 4 GPUs: tensor parallel (every rank runs
every request, fused TP reduce points), expert parallel (each request on one rank,
experts sharded, fused EP exchange, idle ranks run the MoE exchange alone) and the two
combined (attention TP inside data-parallel groups, experts over every rank).

The stage's leader runs in this process on GPU 0 and spawns the follower on GPU 1.
Every generated token must be a greedy choice of the single-GPU model: its logit,
teacher-forced on one GPU, is within a bf16 tolerance of the row's maximum.
"""
import asyncio

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]

OVR = {"thinker": {"num_layers": 2}}


def _check_greedy(reqs, tol=0.08):
    from sglang_omni_b200.models.qwen3_omni import loader
    from tests.test_ar_engine import full_logits

    model = loader.get_thinker("random", torch.device("cuda", 0), OVR)
    for r in reqs:
        seq = list(r.prompt_ids) + list(r.output_ids)
        lg = full_logits(model, seq, torch.device("cuda", 0))
        for i, tok in enumerate(r.output_ids):
            row = lg[len(r.prompt_ids) - 1 + i]
            assert row[tok] >= row.max() - tol, (r.rid, i, float(row.max() - row[tok]))


@pytest.mark.parametrize("kind", ["tp", "ep", "tpep"])
def test_thinker_stage_group_two_gpus(kind):
    """tpep: attention TP over both GPUs combined with expert-parallel MoE over both (one
    data-parallel group; the owned rows of each TP rank are dispatched once)."""
    from sglang_omni_b200.engines.ar import ARRequest
    from sglang_omni_b200.models.qwen3_omni.pipeline.stages import create_thinker_executor
    from sglang_omni_b200.sampling_params import SamplingParams

    sizes = {"tp": {"tp_size": 2}, "ep": {"ep_size": 2}, "tpep": {"tp_size": 2, "ep_size": 2}}[kind]
    ex = create_thinker_executor(model_path="random", device="cuda:0", max_batch=8, max_context=512,
                                 max_prefill_tokens=512, overrides=OVR, **sizes)
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(0, 151000, (n,), generator=g).tolist() for n in (37, 80, 5, 120, 64)]

    async def main():
        ex.engine.start()
        try:
            reqs = [ARRequest(rid=f"{kind}{i}", prompt_ids=p, sampling=SamplingParams(temperature=0.0,
                                                                                      ignore_eos=True),
                              max_new_tokens=6) for i, p in enumerate(prompts)]
            outs = await asyncio.gather(*[ex.engine.generate(r.rid, r) for r in reqs])
            late = ARRequest(rid=f"{kind}-late", prompt_ids=prompts[0], max_new_tokens=3,
                             sampling=SamplingParams(temperature=0.0, ignore_eos=True))
            outs.append(await ex.engine.generate(late.rid, late))
            return outs
        finally:
            ex.engine.stop()

    outs = asyncio.run(main())
    assert [len(r.output_ids) for r in outs] == [6] * 5 + [3]
    if kind == "ep":
        assert ex.engine.threaded.served_remote > 0
    from sglang_omni_b200.ops._ext import check_status

    check_status(torch.device("cuda", 0))
    _check_greedy(outs)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_thinker_stage_tp2_ep4_four_gpus():
    """Two data-parallel groups of 2 TP ranks, 4 expert-parallel ranks; an idle group runs the
    MoE exchange alone while the other serves."""
    from sglang_omni_b200.engines.ar import ARRequest
    from sglang_omni_b200.models.qwen3_omni.pipeline.stages import create_thinker_executor
    from sglang_omni_b200.sampling_params import SamplingParams

    ex = create_thinker_executor(model_path="random", device="cuda:0", max_batch=8, max_context=512,
                                 max_prefill_tokens=512, overrides=OVR, tp_size=2, ep_size=4)
    g = torch.Generator().manual_seed(8)
    prompts = [torch.randint(0, 151000, (n,), generator=g).tolist() for n in (37, 80, 5, 120, 64)]

    async def main():
        ex.engine.start()
        try:
            reqs = [ARRequest(rid=f"g{i}", prompt_ids=p, sampling=SamplingParams(temperature=0.0, ignore_eos=True),
                              max_new_tokens=6) for i, p in enumerate(prompts)]
            outs = await asyncio.gather(*[ex.engine.generate(r.rid, r) for r in reqs])
            late = ARRequest(rid="g-late", prompt_ids=prompts[1], max_new_tokens=3,
                             sampling=SamplingParams(temperature=0.0, ignore_eos=True))
            outs.append(await ex.engine.generate(late.rid, late))
            return outs
        finally:
            ex.engine.stop()

    outs = asyncio.run(main())
    assert [len(r.output_ids) for r in outs] == [6] * 5 + [3]
    assert ex.engine.threaded.served_remote > 0 and ex.engine.threaded.served_local > 0
    from sglang_omni_b200.ops._ext import check_status

    check_status(torch.device("cuda", 0))
    _check_greedy(outs)
