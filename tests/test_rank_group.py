"""Stage rank groups on CPU (the plumbing of tensor / expert parallel stages).

The toy decoder stage is served by a group of two processes built from a YAML
config: in ``replica`` mode both ranks run every request in lock step (the TP
protocol: the leader publishes each iteration's new requests, only the leader
answers); in ``dp`` mode each request runs on one rank and the follower's tokens
come back through the leader (the EP protocol: per-iteration reports, idle
ranks keep stepping while another rank has work).  Greedy outputs must equal
the single-process pipeline's.  A follower that dies fails the in-flight
requests instead of hanging them.
"""
import asyncio
import os
import signal

import pytest
import torch
import yaml

from sglang_omni_b200.client import Client, GenerateRequest, SamplingParams
from sglang_omni_b200.config import PipelineRunner, compile_pipeline
from sglang_omni_b200.config.manager import ConfigManager
from sglang_omni_b200.models.toy.config import ToyPipelineConfig


def _prompts(n=6, L=24):
    g = torch.Generator().manual_seed(1)
    return torch.randint(0, 1000, (n, L), generator=g).tolist()


async def _run(cfg, prompts, max_tokens=12):
    coord, stages = compile_pipeline(cfg)
    async with PipelineRunner(coord, stages):
        client = Client(coord)

        async def one(i):
            req = GenerateRequest(prompt_token_ids=prompts[i], sampling=SamplingParams(temperature=0.0),
                                  max_tokens=max_tokens, stream=True)
            toks = []
            async for ch in client.generate(req):
                if ch.finish_reason is None:
                    toks += ch.token_ids
            return toks

        return await asyncio.gather(*[one(i) for i in range(len(prompts))])


def _group_cfg(tmp_path, mode, size=2, tp=1):
    base = ToyPipelineConfig()
    d = base.model_dump()
    for st in d["stages"]:
        if st["name"] == "decoder":
            st["executor"]["args"].update({"group_mode": mode, "group_size": size, "group_tp": tp})
    p = tmp_path / f"toy_{mode}_{size}_{tp}.yaml"
    p.write_text(yaml.safe_dump(d))
    return ConfigManager.from_file(str(p))


@pytest.mark.parametrize("mode", ["replica", "dp"])
def test_two_rank_stage_group_from_yaml_matches_single_process(tmp_path, mode):
    prompts = _prompts()
    ref = asyncio.run(_run(ToyPipelineConfig(), prompts))
    cfg = _group_cfg(tmp_path, mode)
    outs = asyncio.run(_run(cfg, prompts))
    assert outs == ref
    assert all(len(o) == 12 for o in outs)


def test_four_rank_group_of_two_lockstep_pairs_matches_single_process(tmp_path):
    """The plumbing of attention TP x expert parallel stages: 4 ranks in two data-parallel
    groups of 2 lock-step ranks; requests spread over the groups, every rank of a group runs
    them, the group's first rank reports the tokens."""
    prompts = _prompts()
    ref = asyncio.run(_run(ToyPipelineConfig(), prompts))
    outs = asyncio.run(_run(_group_cfg(tmp_path, "dp", size=4, tp=2), prompts))
    assert outs == ref


def test_rank_group_dp_spreads_requests_and_survives_idle_ranks():
    """With more requests than one rank's share, both ranks serve some; a request that
    arrives while the other rank is idle still completes (idle ranks keep stepping)."""
    from sglang_omni_b200.models.toy.config import create_toy_decoder_executor

    ex = create_toy_decoder_executor(group_mode="dp", group_size=2)
    threaded = ex.engine.threaded

    async def main():
        from sglang_omni_b200.engines.ar import ARRequest

        ex.engine.start()
        try:
            reqs = [ARRequest(rid=f"q{i}", prompt_ids=p, sampling=SamplingParams(temperature=0.0), max_new_tokens=8)
                    for i, p in enumerate(_prompts(5))]
            outs = await asyncio.gather(*[ex.engine.generate(r.rid, r) for r in reqs])
            assert all(len(o.output_ids) == 8 for o in outs)
            # a late request after everything drained
            late = ARRequest(rid="late", prompt_ids=_prompts(1)[0], sampling=SamplingParams(temperature=0.0),
                             max_new_tokens=4)
            r = await ex.engine.generate("late", late)
            assert len(r.output_ids) == 4
        finally:
            ex.engine.stop()

    asyncio.run(main())
    assert threaded.served_remote > 0 and threaded.served_local > 0


def test_rank_group_follower_death_fails_requests():
    from sglang_omni_b200.engines.ar import ARRequest
    from sglang_omni_b200.models.toy.config import create_toy_decoder_executor

    ex = create_toy_decoder_executor(group_mode="dp", group_size=2)

    async def main():
        ex.engine.start()
        try:
            await ex.engine.generate("warm", ARRequest(rid="warm", prompt_ids=[1, 2, 3], max_new_tokens=2,
                                                       sampling=SamplingParams(temperature=0.0)))
            os.kill(ex.engine.threaded.rg.procs[0].pid, signal.SIGKILL)
            reqs = [ARRequest(rid=f"d{i}", prompt_ids=p, sampling=SamplingParams(temperature=0.0),
                              max_new_tokens=64) for i, p in enumerate(_prompts(4))]
            res = await asyncio.wait_for(asyncio.gather(*[ex.engine.generate(r.rid, r) for r in reqs],
                                                        return_exceptions=True), timeout=60)
            assert any(isinstance(x, Exception) for x in res)
        finally:
            ex.engine.stop()

    asyncio.run(main())


def test_host_subgroups_share_one_store():
    """Data-parallel TP subgroups of a 4-rank host group (ranks {0, 1} and {2, 3}) over the same
    TCP store: each subgroup's all-gather / barrier sees only its members, concurrently."""
    import socket
    import threading

    from sglang_omni_b200.parallel.hostgroup import HostGroup

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out, errs = {}, []

    def rank(r):
        try:
            g = HostGroup("127.0.0.1", port, r, 4, timeout_s=30)
            members = [0, 1] if r < 2 else [2, 3]
            sub = g.subgroup(members, f"tp{r // 2}")
            got = sub.all_gather_object(f"r{r}")
            sub.barrier()
            everyone = g.all_gather_object(r * 10)
            out[r] = (sub.rank, sub.world, got, everyone)
        except Exception as exc:   # reported to the test thread
            errs.append(repr(exc))

    ts = [threading.Thread(target=rank, args=(r,)) for r in range(4)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(60)
    assert not errs, errs
    assert out[0][:3] == (0, 2, ["r0", "r1"]) and out[1][:3] == (1, 2, ["r0", "r1"])
    assert out[2][:3] == (0, 2, ["r2", "r3"]) and out[3][:3] == (1, 2, ["r2", "r3"])
    assert all(v[3] == [0, 10, 20, 30] for v in out.values())
