"""PipelineConfig -> runtime objects.

Steps (sglang_omni/config/compiler.py:23-366): apply stage fusion, allocate
control endpoints, build the Coordinator, then every Stage: executor(s) from
their factories (``model_path`` / ``gpu_id`` / ``device`` injected when the
factory's signature asks for them), ``get_next`` routing, the input handler,
the relay and data plane, and the stream wiring (senders get their targets,
receivers get a StreamQueue that doubles as their executors' mailbox).
"""
from __future__ import annotations

import inspect
import os
import uuid
from dataclasses import dataclass
from typing import Any

from ..executors import create_fused_executor
from ..pipeline.control_plane import StageControlPlane
from ..pipeline.coordinator import Coordinator
from ..pipeline.stage.input import AggregatedInput, DirectInput
from ..pipeline.stage.runtime import Stage
from ..pipeline.stage.stream_queue import StreamQueue
from ..pipeline.worker.data_plane import DataPlaneAdapter
from ..pipeline.worker.runtime import Worker
from ..relay import create_relay
from ..utils.misc import import_string
from .schema import PipelineConfig, StageConfig


@dataclass
class Endpoints:
    stages: dict[str, str]
    completion: str
    abort: str


def allocate_endpoints(cfg: PipelineConfig, stage_names: list[str], run_id: str | None = None,
                       multiprocess: bool = True) -> Endpoints:
    run_id = run_id or uuid.uuid4().hex[:10]
    ep = cfg.endpoints
    scheme = ep.scheme if ep.scheme != "auto" else ("ipc" if multiprocess else "local")
    if scheme == "local":
        stages = {n: f"local://{run_id}/{n}" for n in stage_names}
        completion = f"local://{run_id}/_completion"
        abort = f"local://{run_id}/_abort"
    elif scheme == "ipc":
        base = os.path.join(ep.base_path, run_id)
        os.makedirs(base, exist_ok=True)
        stages = {n: f"ipc://{base}/{n}.sock" for n in stage_names}
        completion = cfg.completion_endpoint or f"ipc://{base}/_completion.sock"
        abort = cfg.abort_endpoint or f"ipc://{base}/_abort.sock"
    else:
        port = ep.base_port
        stages = {}
        for n in stage_names:
            stages[n] = f"tcp://127.0.0.1:{port}"
            port += 1
        completion = cfg.completion_endpoint or f"tcp://127.0.0.1:{port}"
        abort = cfg.abort_endpoint or f"tcp://127.0.0.1:{port + 1}"
    return Endpoints(stages, completion, abort)


def _call_factory(factory_path: str, args: dict, model_path: str, gpu_id: int | None):
    factory = import_string(factory_path)
    kwargs = dict(args)
    try:
        params = inspect.signature(factory).parameters
    except (TypeError, ValueError):
        params = {}
    if "model_path" in params and "model_path" not in kwargs:
        from ..models.model_path import resolve_model_path

        kwargs["model_path"] = resolve_model_path(model_path)
    if gpu_id is not None:
        if "gpu_id" in params and "gpu_id" not in kwargs:
            kwargs["gpu_id"] = gpu_id
        if "device" in params and "device" not in kwargs:
            kwargs["device"] = f"cuda:{gpu_id}"
    return factory(**kwargs)


def build_fused_executor(executors: list[dict], names: list[str] | None = None, model_path: str = "",
                         gpu_id: int | None = None):
    built = [_call_factory(e["factory"], e.get("args", {}), model_path, gpu_id) for e in executors]
    return create_fused_executor(built, names)


def _wrap_get_next(fn, name_map: dict[str, str]):
    def get_next(request_id, payload):
        nxt = fn(request_id, payload)
        if nxt is None:
            return None
        if isinstance(nxt, str):
            return name_map.get(nxt, nxt)
        return [name_map.get(n, n) for n in nxt]

    return get_next


def resolve_relay_backend(cfg: PipelineConfig, multiprocess: bool) -> str:
    if cfg.relay_backend == "auto":
        return "shm" if multiprocess else "inproc"
    if cfg.relay_backend in ("nixl", "mooncake"):
        raise ValueError(f"relay backend {cfg.relay_backend!r} targets multi-node RDMA fabrics and is not built "
                         f"into this single-node runtime; use nccl, cuda_ipc, shm or inproc")
    return cfg.relay_backend


def build_stage(cfg: PipelineConfig, s: StageConfig, endpoints: Endpoints, name_map: dict[str, str],
                stream_receivers: set[str], stage_id: int, multiprocess: bool = False,
                gpu_id: int | None = None, relay_ranks: dict[str, int] | None = None) -> Stage:
    if gpu_id is None and s.name in cfg.gpu_placement:
        gpu_id = cfg.gpu_placement[s.name]
    backend = resolve_relay_backend(cfg, multiprocess)
    relay_kwargs = s.relay.model_dump()
    if backend in ("nccl", "cuda_ipc") and relay_kwargs.get("device", "cpu") == "cpu":
        relay_kwargs["device"] = f"cuda:{gpu_id or 0}"
    relay = create_relay(backend, **relay_kwargs)
    cp = StageControlPlane(s.name, endpoints.stages[s.name], endpoints.completion, endpoints.abort)
    data_plane = DataPlaneAdapter(relay, relay_kwargs.get("device", "cpu"))
    if s.input_handler.type == "aggregated":
        merge = import_string(s.input_handler.merge_fn) if s.input_handler.merge_fn else None
        handler = AggregatedInput(s.input_handler.sources or [], merge)
    else:
        handler = DirectInput()
    sq = StreamQueue(max_pending=4096) if s.name in stream_receivers else None
    stage = Stage(s.name, cp, data_plane, handler, sq)
    get_next = _wrap_get_next(import_string(s.get_next), name_map)
    targets = [(name_map.get(t.to_stage, t.to_stage), t.bootstrap) for t in s.stream_to]
    for _ in range(s.num_workers):
        if s.executor.factory.endswith("build_fused_executor"):
            ex = build_fused_executor(model_path=cfg.model_path, gpu_id=gpu_id, **s.executor.args)
        else:
            ex = _call_factory(s.executor.factory, s.executor.args, cfg.model_path, gpu_id)
        w = Worker(s.name, ex, get_next, data_plane, cp, endpoints.stages, targets, stage_id, relay_ranks)
        stage.add_worker(w)
    return stage


def compile_pipeline(cfg: PipelineConfig, run_id: str | None = None) -> tuple[Coordinator, list[Stage]]:
    """Single-process build: every stage in this process (zero-copy in-process relay by default)."""
    stages_cfg, name_map, entry = cfg.apply_fusion()
    names = [s.name for s in stages_cfg]
    endpoints = allocate_endpoints(cfg, names, run_id, multiprocess=False)
    terminals = [name_map.get(t, t) for t in cfg.terminal_stages]
    coordinator = Coordinator(endpoints.completion, endpoints.abort, entry, terminals,
                              request_timeout_s=cfg.request_timeout_s)
    receivers = {name_map.get(t.to_stage, t.to_stage) for s in stages_cfg for t in s.stream_to}
    stages = []
    for i, s in enumerate(stages_cfg):
        stages.append(build_stage(cfg, s, endpoints, name_map, receivers, i))
        coordinator.register_stage(s.name, endpoints.stages[s.name])
    return coordinator, stages
