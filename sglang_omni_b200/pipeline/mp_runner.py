"""One OS process per stage (stage-level MPMD across GPUs).

Each child pins its GPU from ``gpu_placement`` before touching CUDA, rebuilds
its stage from the (picklable) config, binds its control socket, signals
readiness and runs until shutdown.  The parent hosts the coordinator, waits
for every child with a bounded startup timeout (rolling back on failure),
and monitors liveness: a dead stage fails the pipeline instead of leaving
requests hanging -- or, with ``restart``, the runner fails the requests in
flight, starts a new process for that stage on the same endpoints and keeps
serving (the reference has no recovery; this is the optional one of the plan).  With ``relay_backend: nccl`` the stage processes form one
torch.distributed NCCL group (rank = stage index) for point-to-point relays.

Reference counterpart: sglang_omni/pipeline/mp_runner.py:203-486.
"""
from __future__ import annotations

import asyncio
import logging
import multiprocessing as mp
import os
import socket
import time
import traceback
import uuid

from ..config.compiler import allocate_endpoints, build_stage, resolve_relay_backend
from ..config.schema import PipelineConfig
from .coordinator import Coordinator

log = logging.getLogger(__name__)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _stage_process_entry(cfg_dict: dict, cfg_cls_path: str | None, stage_index: int, run_id: str, ready, failed,
                         dist_env: dict | None):
    try:
        cfg_cls = PipelineConfig
        if cfg_cls_path:
            from ..utils.misc import import_string
            cfg_cls = import_string(cfg_cls_path)
        cfg = cfg_cls(**cfg_dict)
        stages_cfg, name_map, _ = cfg.apply_fusion()
        s = stages_cfg[stage_index]
        gpu = cfg.gpu_placement.get(s.name)
        group_stage = any(int(s.executor.args.get(k, 1) or 1) > 1 for k in ("tp_size", "ep_size"))
        if gpu is not None and not group_stage:
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = visible.split(",")[gpu] if visible else str(gpu)
            os.environ.setdefault("OMNI_VISIBLE_DEVICES_ORIG", visible or "")
            os.environ["CUDA_VISIBLE_DEVICES"] = phys
        # a stage served by a rank group (tp_size / ep_size > 1) keeps every GPU visible: its ranks
        # map each other's buffers through CUDA IPC; it runs on GPU `gpu` of the pipeline's set
        import torch  # noqa: F401  (after the device mask)

        local_gpu = (gpu if group_stage else 0) if gpu is not None else None
        relay_ranks = None
        if dist_env is not None:
            os.environ.update({k: str(v) for k, v in dist_env.items()})
            import torch.distributed as dist
            from datetime import timedelta

            torch.cuda.set_device(local_gpu or 0)
            dist.init_process_group("nccl", rank=stage_index, world_size=len(stages_cfg),
                                    timeout=timedelta(seconds=120))
            relay_ranks = {st.name: i for i, st in enumerate(stages_cfg)}
            # every pair of stage processes connects once, in one global order, before any stage
            # sends (a first send would otherwise block its host thread until the peer receives)
            from ..relay.nccl import NcclRelay

            NcclRelay(rank=stage_index, world_size=len(stages_cfg), device=f"cuda:{local_gpu or 0}").warmup_all()
        endpoints = allocate_endpoints(cfg, [st.name for st in stages_cfg], run_id)
        receivers = {name_map.get(t.to_stage, t.to_stage) for st in stages_cfg for t in st.stream_to}
        stage = build_stage(cfg, s, endpoints, name_map, receivers, stage_index, multiprocess=True,
                            gpu_id=local_gpu, relay_ranks=relay_ranks)

        async def main():
            await stage.start()
            ready.set()
            await stage.run()
            await stage.stop()

        asyncio.run(main())
    except BaseException:
        traceback.print_exc()
        failed.set()
        raise SystemExit(1)


class MultiProcessPipelineRunner:
    def __init__(self, cfg: PipelineConfig, startup_timeout: float | None = None, monitor_interval: float = 5.0,
                 restart: bool | list[str] = False, max_restarts: int = 3):
        """``restart``: True (every stage that can be restarted) or the names of such stages.
        A stage can be restarted unless the pipeline relays over NCCL (a new process cannot
        join the stage processes' group) or a rank group serves it (tp_size / ep_size > 1).
        A restart fails every request in flight: the runner does not know which of them held
        state in the dead stage.  After ``max_restarts`` restarts of one stage its next death
        stops the pipeline."""
        self.cfg = cfg
        self.restart = restart
        self.max_restarts = max_restarts
        self.restarts: dict[str, int] = {}
        self._spawn_args: dict[str, tuple] = {}
        self.startup_timeout = startup_timeout or float(os.environ.get("SGLANG_OMNI_STARTUP_TIMEOUT", "600"))
        self.monitor_interval = monitor_interval
        self.run_id = uuid.uuid4().hex[:10]
        self.procs: list[mp.Process] = []
        self.coordinator: Coordinator | None = None
        self._monitor: asyncio.Task | None = None
        self._loop_task: asyncio.Task | None = None
        self.failed_stage: str | None = None

    async def start(self):
        stages_cfg, name_map, entry = self.cfg.apply_fusion()
        names = [s.name for s in stages_cfg]
        endpoints = allocate_endpoints(self.cfg, names, self.run_id)
        terminals = [name_map.get(t, t) for t in self.cfg.terminal_stages]
        self.coordinator = Coordinator(endpoints.completion, endpoints.abort, entry, terminals,
                                       request_timeout_s=self.cfg.request_timeout_s)
        await self.coordinator.start()
        for n in names:
            self.coordinator.register_stage(n, endpoints.stages[n])
        ctx = mp.get_context("spawn")
        dist_env = None
        if resolve_relay_backend(self.cfg, True) == "nccl":
            dist_env = {"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": _free_port()}
        cls = type(self.cfg)
        cls_path = None if cls is PipelineConfig else f"{cls.__module__}.{cls.__qualname__}"
        events = []
        self._ctx, self._dist = ctx, dist_env
        for i, n in enumerate(names):
            self._spawn_args[n] = (i, cls_path)
            p, ready, failed = self._spawn(n)
            self.procs.append(p)
            events.append((n, p, ready, failed))
        deadline = time.monotonic() + self.startup_timeout
        for n, p, ready, failed in events:
            while not ready.is_set():
                if failed.is_set() or not p.is_alive():
                    self._kill_all()
                    raise RuntimeError(f"stage {n!r} died during startup")
                if time.monotonic() > deadline:
                    self._kill_all()
                    raise TimeoutError(f"stage {n!r} not ready after {self.startup_timeout:.0f}s")
                await asyncio.sleep(0.05)
        await asyncio.sleep(0.1)
        self._loop_task = self.coordinator.start_completion_loop()
        self._monitor = asyncio.ensure_future(self._monitor_children(names))

    def _spawn(self, name: str):
        i, cls_path = self._spawn_args[name]
        ready, failed = self._ctx.Event(), self._ctx.Event()
        p = self._ctx.Process(target=_stage_process_entry, name=f"stage-{name}",
                              args=(self.cfg.model_dump(), cls_path, i, self.run_id, ready, failed, self._dist),
                              daemon=True)
        p.start()
        return p, ready, failed

    def restartable(self, name: str) -> bool:
        if not self.restart or self._dist is not None:
            return False
        if isinstance(self.restart, (list, tuple, set)) and name not in self.restart:
            return False
        st = next(s for s in self.cfg.apply_fusion()[0] if s.name == name)
        return not any(int(st.executor.args.get(k, 1) or 1) > 1 for k in ("tp_size", "ep_size"))

    def _fail_in_flight(self, why: str):
        for rid in list(self.coordinator._reqs):
            self.coordinator._finish(rid, self.coordinator._reqs[rid].info.state.__class__.FAILED,
                                     exc=RuntimeError(why))

    async def _restart(self, idx: int, name: str, exitcode) -> bool:
        """Replaces a dead stage process; False if the new one did not come up in time."""
        self.restarts[name] = self.restarts.get(name, 0) + 1
        log.error("stage process %s exited with %s; failing requests in flight and restarting it (%d of %d)",
                  name, exitcode, self.restarts[name], self.max_restarts)
        self._fail_in_flight(f"stage {name} died and was restarted")
        p, ready, failed = self._spawn(name)
        self.procs[idx] = p
        deadline = time.monotonic() + self.startup_timeout
        while not ready.is_set():
            if failed.is_set() or not p.is_alive() or time.monotonic() > deadline:
                return False
            await asyncio.sleep(0.05)
        return True

    async def _monitor_children(self, names):
        while True:
            await asyncio.sleep(self.monitor_interval)
            for idx, (n, p) in enumerate(zip(names, list(self.procs))):
                if not p.is_alive():
                    if self.restartable(n) and self.restarts.get(n, 0) < self.max_restarts:
                        if await self._restart(idx, n, p.exitcode):
                            continue
                    self.failed_stage = n
                    log.error("stage process %s exited with %s; stopping the pipeline", n, p.exitcode)
                    self.coordinator.running = False
                    # fail every in-flight request
                    for rid in list(self.coordinator._reqs):
                        self.coordinator._finish(rid, self.coordinator._reqs[rid].info.state.__class__.FAILED,
                                                 exc=RuntimeError(f"stage {n} died"))
                    return

    def _kill_all(self):
        for p in self.procs:
            if p.is_alive():
                p.terminate()
        for p in self.procs:
            p.join(timeout=5)
            if p.is_alive():
                p.kill()

    async def stop(self):
        if self._monitor is not None:
            self._monitor.cancel()
        if self.coordinator is not None:
            await self.coordinator.stop()
        for p in self.procs:
            p.join(timeout=10)
        self._kill_all()

    async def __aenter__(self):
        await self.start()
        return self

    async def __aexit__(self, *exc):
        await self.stop()
