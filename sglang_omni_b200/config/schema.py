"""Pipeline configuration schema.

Field names, defaults and validation follow the reference
(sglang_omni/config/schema.py:11-222) so YAML written for it loads here:
unique stage names, entry stage defined, aggregated sources and stream_to
targets exist, fused groups adjacent and in order.  Additions: relay backends
``inproc`` / ``cuda_ipc`` / ``auto`` (in-process when every stage shares the
process, shm otherwise) and per-stage parallel layout in executor args.
"""
from __future__ import annotations

from typing import Any, Literal

from pydantic import BaseModel, ConfigDict, Field


class ExecutorConfig(BaseModel):
    model_config = ConfigDict(extra="forbid")
    factory: str
    args: dict[str, Any] = Field(default_factory=dict)


class InputHandlerConfig(BaseModel):
    model_config = ConfigDict(extra="forbid")
    type: Literal["direct", "aggregated"] = "direct"
    sources: list[str] | None = None
    merge_fn: str | None = None


class RelayConfig(BaseModel):
    model_config = ConfigDict(extra="forbid")
    slot_size_mb: int = 512
    credits: int = 2
    rank: int | None = None
    world_size: int | None = None
    device: str = "cpu"


class StreamTargetConfig(BaseModel):
    model_config = ConfigDict(extra="forbid")
    to_stage: str
    bootstrap: bool = True


class StageConfig(BaseModel):
    model_config = ConfigDict(extra="forbid")
    name: str
    executor: ExecutorConfig
    get_next: str
    input_handler: InputHandlerConfig = Field(default_factory=InputHandlerConfig)
    relay: RelayConfig = Field(default_factory=RelayConfig)
    num_workers: int = 1
    stream_to: list[StreamTargetConfig] = Field(default_factory=list)


class EndpointsConfig(BaseModel):
    model_config = ConfigDict(extra="forbid")
    scheme: Literal["auto", "ipc", "tcp", "local"] = "auto"  # auto: local in one process, else ipc
    base_path: str = "/tmp/sglang_omni_b200"
    base_port: int = 16000


class PipelineConfig(BaseModel):
    model_config = ConfigDict(extra="forbid")

    model_path: str
    entry_stage: str
    stages: list[StageConfig]
    name: str = "model"
    terminal_stages: list[str] = Field(default_factory=list)
    relay_backend: Literal["auto", "inproc", "shm", "nccl", "cuda_ipc", "nixl", "mooncake"] = "auto"
    fused_stages: list[list[str]] = Field(default_factory=list)
    endpoints: EndpointsConfig = Field(default_factory=EndpointsConfig)
    gpu_placement: dict[str, int] = Field(default_factory=dict)
    completion_endpoint: str | None = None
    abort_endpoint: str | None = None
    config_cls: str | None = None
    # a request not completed this long after submission fails with a timeout (None: no deadline)
    request_timeout_s: float | None = None

    def model_post_init(self, __context: Any = None) -> None:
        problems = self.problems()
        if problems:
            raise ValueError(f"invalid pipeline config {self.name!r}: " + "; ".join(problems))
        if self.config_cls is None or self.config_cls == "PipelineConfig":
            self.config_cls = self.__class__.__name__

    @staticmethod
    def from_dict(data: dict[str, Any]) -> "PipelineConfig":
        return PipelineConfig(**data)

    def stage(self, name: str) -> StageConfig:
        for s in self.stages:
            if s.name == name:
                return s
        raise KeyError(name)

    def problems(self) -> list[str]:
        """Every inconsistency of the config, in one pass (empty when it is usable).

        The same conditions make a config unusable as in the reference's schema
        (sglang_omni/config/schema.py:105-175): names referenced by the entry, routing,
        aggregation, streaming, terminal and fusion fields must be stages; stage names are
        unique; every stage has a factory, a routing function and a worker; a fused group
        lists two or more adjacent stages in pipeline order, each stage in one group."""
        out: list[str] = []
        order = {}
        for i, s in enumerate(self.stages):
            if s.name in order:
                out.append(f"two stages are named {s.name!r}")
            order.setdefault(s.name, i)
        if not self.model_path:
            out.append("no model_path")
        if not self.stages:
            out.append("no stages")
        elif self.entry_stage not in order:
            out.append(f"entry stage {self.entry_stage!r} is not one of the stages {list(order)}")
        for s in self.stages:
            lacks = [what for what, ok in (("an executor factory", s.executor.factory), ("get_next", s.get_next),
                                           ("a worker", s.num_workers >= 1)) if not ok]
            if lacks:
                out.append(f"stage {s.name!r} lacks " + ", ".join(lacks))
            refs = [("stream target", st.to_stage) for st in s.stream_to]
            if s.input_handler.type == "aggregated":
                refs += [("aggregation source", src) for src in s.input_handler.sources or []]
            out += [f"stage {s.name!r}: {what} {ref!r} is not a stage" for what, ref in refs if ref not in order]
        out += [f"terminal stage {t!r} is not a stage" for t in self.terminal_stages if t not in order]
        grouped: set[str] = set()
        for group in self.fused_stages or []:
            where = [order.get(n) for n in group]
            if len(group) < 2:
                out.append(f"fused group {group} has fewer than two stages")
            if None in where:
                out.append(f"fused group {group} names a stage that does not exist")
                continue
            if where != list(range(where[0], where[0] + len(where))):
                out.append(f"fused group {group} is not a run of neighbouring stages in pipeline order")
            again = grouped.intersection(group)
            if again:
                out.append(f"stages {sorted(again)} are in more than one fused group")
            grouped.update(group)
        return out

    def apply_fusion(self) -> tuple[list[StageConfig], dict[str, str], str]:
        """Collapses each fused group into one stage named after its last member."""
        by_name = {s.name: s for s in self.stages}
        name_map = {n: n for n in by_name}
        group_by_last: dict[str, list[str]] = {}
        for g in self.fused_stages or []:
            group_by_last[g[-1]] = g
            for n in g:
                name_map[n] = g[-1]
        out: list[StageConfig] = []
        for s in self.stages:
            if name_map[s.name] != s.name:
                continue
            if s.name in group_by_last:
                g = group_by_last[s.name]
                first = by_name[g[0]]
                out.append(StageConfig(
                    name=s.name,
                    executor=ExecutorConfig(
                        factory="sglang_omni_b200.config.compiler.build_fused_executor",
                        args={"executors": [{"factory": by_name[n].executor.factory, "args": by_name[n].executor.args}
                                            for n in g], "names": list(g)}),
                    get_next=s.get_next, input_handler=first.input_handler, relay=first.relay,
                    num_workers=first.num_workers, stream_to=first.stream_to))
            else:
                out.append(s)
        return out, name_map, name_map[self.entry_stage]
