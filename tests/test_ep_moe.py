"""Expert-parallel MoE over peer memory (one process per GPU): the EP layer
(local routing, dispatch with system-atomic reservations into the owners'
receive segments, the flag wait inside the w13 grouped GEMM, the w2 epilogue
storing rows into their source ranks' slots, the combine waiting on the
owners' flags) must match the dense fp32 MoE of the same weights, eagerly and
replayed from a CUDA graph.  A world-of-one group runs on one GPU (every peer
pointer is this GPU's own buffer), the 2-GPU case across NVLink."""
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


def _run_world1():
    """The whole EP layer with a group of one (loopback through this GPU's own buffer)."""
    import torch.distributed as dist

    from sglang_omni_b200.ops._ext import check_status
    from sglang_omni_b200.ops.moe import moe_ref
    from sglang_omni_b200.parallel import EPMoE

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)
    try:
        E, k, H, I = 16, 4, 256, 128
        g = torch.Generator().manual_seed(1)
        router = (torch.randn(E, H, generator=g) * 0.5).bfloat16()
        w13 = (torch.randn(E, 2 * I, H, generator=g) * 0.05).bfloat16()
        w2 = (torch.randn(E, H, I, generator=g) * 0.05).bfloat16()
        ep = EPMoE(E, k, H, I, max_tokens=96, device=dev)
        r_dev, w13_d, w2_d = router.to(dev), w13.to(dev), w2.to(dev)
        errs = []
        for T in (37, 0, 96, 5):
            x = (torch.randn(T, H, generator=torch.Generator().manual_seed(20 + T)) * 0.5).bfloat16()
            out = ep.forward(x.to(dev), r_dev, w13_d, w2_d)
            torch.cuda.synchronize()
            check_status(dev)
            if T:
                ref = moe_ref(x, router, w13, w2, k)
                errs.append(float((out.cpu().float() - ref).norm() / ref.norm()))
            assert int(ep.cursor.sum()) == 0, "the w2 GEMM leaves the receive counters cleared"
        # fused add + RMSNorm output and graph replay
        x = (torch.randn(16, H, generator=torch.Generator().manual_seed(99)) * 0.5).bfloat16().to(dev)
        ref = moe_ref(x.cpu(), router, w13, w2, k)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ep.forward(x, r_dev, w13_d, w2_d)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            y = ep.forward(x, r_dev, w13_d, w2_d)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        check_status(dev)
        errs.append(float((y.cpu().float() - ref).norm() / ref.norm()))
        del graph
        ep.close()
        return errs
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_ep_moe_world1_loopback_matches_dense():
    errs = _run_world1()
    assert max(errs) < 0.02, errs


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
