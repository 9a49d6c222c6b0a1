"""Server launcher: single process (all stages in this process) when at most
one distinct GPU is placed, else one process per stage; then Client + app +
uvicorn.  Profiler routes broadcast start / stop to every stage in both modes
(the reference disables them in multi-process mode,
sglang_omni/serve/launcher.py:107-264)."""
from __future__ import annotations

import asyncio
import logging
import os
import socket
import time

from ..client import Client
from ..config import PipelineConfig, PipelineRunner, compile_pipeline
from .openai_api import create_app

log = logging.getLogger(__name__)


def find_available_port(start: int = 8000, host: str = "127.0.0.1", tries: int = 200) -> int:
    for p in range(start, start + tries):
        with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
            try:
                s.bind((host, p))
                return p
            except OSError:
                continue
    raise RuntimeError("no free port")


def _mount_profiler_routes(app, coordinator):
    @app.post("/start_profile")
    async def start_profile(body: dict | None = None):
        run_id = (body or {}).get("run_id") or time.strftime("%Y%m%d-%H%M%S")
        root = os.environ.get("SGLANG_TORCH_PROFILER_DIR", "/tmp/sglang_omni_b200_profiles")
        await coordinator.start_profile(run_id, os.path.join(root, "{run_id}", "{stage}", "trace"))
        return {"run_id": run_id}

    @app.post("/stop_profile")
    async def stop_profile(body: dict | None = None):
        await coordinator.stop_profile((body or {}).get("run_id", ""))
        return {"ok": True}


async def build_server(cfg: PipelineConfig, model_name: str | None = None, tokenizer=None,
                       restart_stages: list[str] | None = None):
    """Returns (app, runner) with the pipeline started.  ``restart_stages`` (multi-process
    pipelines: stages placed on more than one GPU): stages whose process is replaced when it
    dies, instead of stopping the server."""
    gpus = set(cfg.gpu_placement.values())
    if len(gpus) > 1:
        from ..pipeline.mp_runner import MultiProcessPipelineRunner

        runner = MultiProcessPipelineRunner(cfg, restart=list(restart_stages or []))
        await runner.start()
        coordinator = runner.coordinator
    else:
        coordinator, stages = compile_pipeline(cfg)
        runner = PipelineRunner(coordinator, stages)
        await runner.start()
    client = Client(coordinator, tokenizer, model_name or cfg.name)
    app = create_app(client, model_name or cfg.name)
    _mount_profiler_routes(app, coordinator)
    return app, runner


def launch_server(cfg: PipelineConfig, host: str = "0.0.0.0", port: int = 8000, model_name: str | None = None,
                  log_level: str = "info", restart_stages: list[str] | None = None) -> None:
    import uvicorn

    async def main():
        app, runner = await build_server(cfg, model_name, restart_stages=restart_stages)
        server = uvicorn.Server(uvicorn.Config(app, host=host, port=port, log_level=log_level))
        try:
            await server.serve()
        finally:
            await runner.stop()

    asyncio.run(main())
