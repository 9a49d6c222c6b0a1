"""GPU relays between two processes on two GPUs: NCCL point-to-point (send / recv on a
side stream, completion through an event, no host synchronisation on the sender) and
CUDA IPC (interprocess event instead of a sender-side synchronize).  Payloads of several
sizes, produced by a kernel right before the put, must arrive intact."""
import os
import socket

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]

SIZES = [1, 4096, 8192 + 3, 1 << 20, 3 << 20]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _payload(i, n, device):
    g = torch.Generator(device=device).manual_seed(100 + i)
    return torch.randint(0, 255, (n,), dtype=torch.uint8, device=device, generator=g)


def _nccl_worker(rank, port, q, meta_q):
    import asyncio
    import faulthandler
    from datetime import timedelta

    import torch.distributed as dist

    faulthandler.dump_traceback_later(150, exit=True)   # a stuck worker prints where it is and ends
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=2, device_id=torch.device("cuda", rank),
                                timeout=timedelta(seconds=60))
        from sglang_omni_b200.relay.nccl import NcclRelay

        relay = NcclRelay(rank=rank, world_size=2, device=f"cuda:{rank}")
        relay.warmup_all()   # connections first: a first send blocks its host thread until the peer receives

        async def main():
            if rank == 0:
                for i, n in enumerate(SIZES):
                    x = _payload(i, n, "cuda:0") * 1            # produced by a kernel just before the put
                    op = await relay.put_async(x, f"r{i}", dst=1)
                    meta_q.put(op.metadata)
                torch.cuda.synchronize()
                return True
            ok = True
            for i, n in enumerate(SIZES):
                md = meta_q.get(timeout=60)
                op = await relay.get_async(md)
                got = await op.wait_for_completion(30)
                ok &= bool(torch.equal(got.cpu(), _payload(i, n, "cuda:1").cpu()))
            return ok

        res = asyncio.run(main())
        torch.cuda.synchronize()
        q.put((rank, res, None))          # reported before the shutdown collectives
        for i in range(len(SIZES)):
            relay.cleanup(f"r{i}")
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, False, traceback.format_exc()))


def _ipc_worker(rank, q, meta_q, done_q):
    import asyncio

    try:
        torch.cuda.set_device(rank)
        from sglang_omni_b200.relay.ipc import CudaIpcRelay

        relay = CudaIpcRelay(device=f"cuda:{rank}")

        async def main():
            if rank == 0:
                for i, n in enumerate(SIZES):
                    x = _payload(i, n, "cuda:0") * 1
                    op = await relay.put_async(x, f"r{i}")
                    meta_q.put(op.metadata)
                done_q.get(timeout=60)                        # keep the buffers until the receiver copied
                for i in range(len(SIZES)):
                    relay.cleanup(f"r{i}")
                return True
            ok = True
            for i, n in enumerate(SIZES):
                md = meta_q.get(timeout=60)
                op = await relay.get_async(md)
                got = await op.wait_for_completion(30)
                torch.cuda.synchronize()
                ok &= bool(torch.equal(got.to("cuda:1").cpu(), _payload(i, n, "cuda:1").cpu()))
            done_q.put(True)
            return ok

        q.put((rank, asyncio.run(main()), None))
    except Exception:
        import traceback

        q.put((rank, False, traceback.format_exc()))


def _run(target, args_fn):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q, meta_q, extra = ctx.Queue(), ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=target, args=args_fn(r, q, meta_q, extra)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, tb in res:
        assert tb is None, tb
        assert ok, rank


def test_nccl_relay_two_gpus():
    port = _free_port()
    _run(_nccl_worker, lambda r, q, mq, _e: (r, port, q, mq))


def test_cuda_ipc_relay_two_gpus():
    _run(_ipc_worker, lambda r, q, mq, e: (r, q, mq, e))
