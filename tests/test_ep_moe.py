"""Expert-parallel MoE over peer memory on 2+ GPUs (one process per GPU): the EP
layer (local routing, peer-store dispatch into expert-major receive buffers,
grouped GEMMs on the owner, peer-store combine, weighted sum) must match the
dense fp32 MoE of the same weights, eagerly and replayed from a CUDA graph."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=60))
        from sglang_omni_b200.ops._ext import check_status
        from sglang_omni_b200.ops.moe import moe_ref
        from sglang_omni_b200.parallel import EPMoE

        E, k, H, I = 16, 4, 256, 128
        g = torch.Generator().manual_seed(0)
        router = (torch.randn(E, H, generator=g) * 0.5).bfloat16()
        w13 = (torch.randn(E, 2 * I, H, generator=g) * 0.05).bfloat16()
        w2 = (torch.randn(E, H, I, generator=g) * 0.05).bfloat16()
        El = E // world
        sl = slice(rank * El, (rank + 1) * El)
        ep = EPMoE(E, k, H, I, max_tokens=64, device=dev)
        r_dev, w13_l, w2_l = router.to(dev), w13[sl].contiguous().to(dev), w2[sl].contiguous().to(dev)
        errs = []
        for T in (37 + 5 * rank, 0 if rank == 1 else 3, 64):
            x = (torch.randn(T, H, generator=torch.Generator().manual_seed(10 + rank + T)) * 0.5).bfloat16()
            out = ep.forward(x.to(dev), r_dev, w13_l, w2_l)
            torch.cuda.synchronize()
            check_status(dev)
            if T:
                ref = moe_ref(x, router, w13, w2, k)
                errs.append(float((out.cpu().float() - ref).norm() / ref.norm()))
        # graph capture + replay (same launches, device-side epochs)
        x = (torch.randn(16, H, generator=torch.Generator().manual_seed(99 + rank)) * 0.5).bfloat16().to(dev)
        ref = moe_ref(x.cpu(), router, w13, w2, k)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ep.forward(x, r_dev, w13_l, w2_l)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            y = ep.forward(x, r_dev, w13_l, w2_l)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        check_status(dev)
        errs.append(float((y.cpu().float() - ref).norm() / ref.norm()))
        del graph
        ep.close()
        dist.destroy_process_group()
        q.put((rank, errs, None))
    except Exception as exc:  # report instead of hanging the parent
        import traceback

        q.put((rank, None, traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_moe_matches_dense():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, errs, tb in res:
        assert tb is None, tb
        assert max(errs) < 0.02, (rank, errs)
