"""Rank groups inside one pipeline stage (tensor / expert parallel serving).

A stage whose executor asks for ``tp_size`` or ``ep_size`` > 1 keeps its place
in the pipeline as ONE stage (one control endpoint, one scheduler): the stage
process is rank 0, the *leader*, and spawns one *follower* process per other
GPU of the group.  Every rank builds its shard of the model and a paged engine
of its own; the leader forwards what its scheduler receives:

* ``tp`` (tensor parallel) -- every rank serves every request.  The leader
  publishes each iteration's new requests / aborts and the followers apply them
  at the same iteration, so the identical, deterministic engines step in lock
  step (the fused TP kernels synchronise the data on the device).  Only the
  leader emits results.
* ``ep`` (expert parallel with data-parallel attention) -- each request goes
  to one rank (the least loaded); the MoE layers exchange rows between all
  ranks, so every rank must run a forward whenever any rank does: a rank with
  nothing to schedule runs an idle forward (the MoE exchange of each layer
  with zero tokens).  Followers report, after every iteration, whether they
  still have work and the tokens they produced; the leader routes those to the
  requests' streams and futures.
* ``ep`` with ``tp`` > 1 -- attention tensor parallel inside data-parallel
  groups of ``tp`` consecutive ranks, MoE expert parallel over all ranks: a
  request goes to one group (every rank of it adds the request in the same
  iteration and steps in lock step, as in ``tp``), the group's first rank
  reports its tokens, and idle groups run the idle forward.
* ``replica`` / ``dp`` -- the same protocols without a sharded model (every
  rank holds a full copy; ``dp`` with ``tp`` > 1 has lock-step groups); they run
  on CPU as well and test the plumbing.

Bootstrap (CUDA IPC handles of the symmetric buffers) goes over a TCP store
(``HostGroup``), the per-iteration control over ZMQ (leader PUB -> followers,
followers PUSH -> leader), the data over NVLink peer memory.

Reference counterparts: SGLang's TP worker processes spawned per scheduler with
``broadcast_pyobj`` of the received requests (the reference hard-wires
``tp_size=1``: sglang_omni/engines/ar/sglang_backend/server_args_builder.py:24-25,
model_worker.py:107-118).
"""
from __future__ import annotations

import copy
import logging
import multiprocessing as mp
import os
import socket
import time
from dataclasses import dataclass, field

import torch

from ..engines.ar.engine import AREngine, ThreadedAREngine
from ..engines.ar.request import ARRequest
from ..utils.misc import import_string

log = logging.getLogger(__name__)

MODES = ("tp", "ep", "replica", "dp")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@dataclass
class GroupSpec:
    """Everything a follower needs to rebuild its rank (picklable)."""
    mode: str
    world: int
    gpus: list = field(default_factory=list)   # GPU index per rank (in the pipeline's visible set); empty = CPU
    builder: str = ""                           # "module.fn": fn(args, rank, world, device, group) -> model
    builder_args: dict = field(default_factory=dict)
    engine_args: dict = field(default_factory=dict)
    kv_pages: int = 0
    host: str = "127.0.0.1"
    store_port: int = 0
    pub_port: int = 0
    pull_port: int = 0
    report_timeout_s: float = 120.0
    tp: int = 1                                 # ranks per data-parallel group (distributing modes)

    @property
    def groups(self) -> int:
        return self.world // self.tp

    def group_of(self, rank: int) -> int:
        return rank // self.tp

    def reports_events(self, rank: int) -> bool:
        """The first rank of a data-parallel group reports its requests' tokens."""
        return self.distributes and rank % self.tp == 0

    def device_of(self, rank: int) -> torch.device:
        return torch.device("cuda", int(self.gpus[rank])) if self.gpus else torch.device("cpu")

    @property
    def sharded(self) -> bool:
        return self.mode in ("tp", "ep")

    @property
    def distributes(self) -> bool:
        """Requests go to one rank each (and results come back from it)."""
        return self.mode in ("ep", "dp")


def _build_rank(spec: GroupSpec, rank: int, device: torch.device):
    from ..engines.ar import KVPool
    from .hostgroup import HostGroup

    group = HostGroup(spec.host, spec.store_port, rank, spec.world, timeout_s=spec.report_timeout_s)
    args = dict(spec.builder_args)
    args.setdefault("tp", spec.tp)
    model = import_string(spec.builder)(args, rank, spec.world, device, group, spec.mode)
    cfg = model.cfg
    pool = KVPool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, spec.kv_pages, device, cfg.dtype)
    eng = AREngine(model, pool, **spec.engine_args)
    return group, model, eng


def _stable_copy(req: ARRequest) -> ARRequest:
    """A picklable copy for another rank: no callbacks, tensors on the CPU."""
    r = copy.copy(req)
    r.on_token = None
    r.extra = {k: v for k, v in req.extra.items() if not callable(v)}
    for name in ("input_embeds", "mm_index", "mm_embeds", "mrope_positions", "ds_positions"):
        t = getattr(r, name)
        if isinstance(t, torch.Tensor):
            setattr(r, name, t.detach().cpu())
    if r.deepstack is not None:
        r.deepstack = [t.detach().cpu() if isinstance(t, torch.Tensor) else t for t in r.deepstack]
    r.output_ids = list(req.output_ids)
    r.pages, r.prefix_nodes = [], []
    return r


def _idle_forward(model, spec: GroupSpec):
    """Every rank runs one forward per iteration of an EP group: the MoE exchange of each layer."""
    if spec.mode == "ep" and hasattr(model, "ep_idle"):
        model.ep_idle()


def _step(eng: AREngine, model, spec: GroupSpec) -> list:
    finished = eng.step()
    if not eng.last_launched:
        _idle_forward(model, spec)
    return finished


def _follower_main(spec: GroupSpec, rank: int):  # pragma: no cover - runs in a spawned process
    import zmq

    if spec.gpus and os.environ.get("OMNI_VISIBLE_DEVICES_ORIG") is not None:
        # a stage process narrowed the mask to its own GPU: every GPU of the group must be visible
        # (CUDA IPC maps the peers' buffers), so restore the pipeline's mask
        orig = os.environ["OMNI_VISIBLE_DEVICES_ORIG"]
        if orig:
            os.environ["CUDA_VISIBLE_DEVICES"] = orig
        else:
            os.environ.pop("CUDA_VISIBLE_DEVICES", None)
    device = spec.device_of(rank)
    if device.type == "cuda":
        torch.cuda.set_device(device)
    ctx = zmq.Context()
    sub = ctx.socket(zmq.SUB)
    sub.setsockopt(zmq.SUBSCRIBE, b"")
    sub.connect(f"tcp://{spec.host}:{spec.pub_port}")
    push = ctx.socket(zmq.PUSH)
    push.connect(f"tcp://{spec.host}:{spec.pull_port}")
    try:
        group, model, eng = _build_rank(spec, rank, device)
        if device.type == "cuda":
            eng.runner.capture_all()
        push.send_pyobj({"ready": rank})
        events: list = []

        def on_token(r, tok, info):
            events.append(("tok", r.rid, int(tok)))

        while True:
            msg = sub.recv_pyobj()
            if msg["kind"] == "stop":
                break
            head = spec.reports_events(rank)
            for kind, dst, x in msg["items"]:
                if dst not in (-1, spec.group_of(rank)):
                    continue
                if kind == "add":
                    if head:
                        x.on_token = on_token
                    try:
                        eng.add_request(x)
                    except Exception as exc:   # the leader rejects the same request (tp) or reports it
                        if head:
                            events.append(("done", x.rid, [], f"error: {exc}"))
                elif kind == "abort":
                    r = eng.requests.get(x)
                    if r is not None and eng.abort(x) and head:
                        events.append(("done", r.rid, list(r.output_ids), r.finish_reason))
            if msg["step"]:
                for r in _step(eng, model, spec):
                    if head:
                        events.append(("done", r.rid, list(r.output_ids), r.finish_reason))
            if spec.distributes:
                push.send_pyobj({"it": msg["it"], "rank": rank, "has_work": eng.has_work(), "events": events})
                events = []
        if device.type == "cuda":
            torch.cuda.synchronize()
        eng.runner.graphs.clear()
        closer = getattr(model, "close_parallel", None)
        if closer is not None:
            closer()
    except BaseException:
        import traceback

        traceback.print_exc()
        try:
            push.send_pyobj({"error": rank, "trace": traceback.format_exc()})
        except Exception:
            pass
        raise SystemExit(1)
    finally:
        sub.close(0)
        push.close(0)
        ctx.term()


class StageRankGroup:
    """Leader side: spawns the followers, builds rank 0 and owns the control sockets."""

    def __init__(self, spec: GroupSpec):
        assert spec.mode in MODES, f"unknown rank-group mode {spec.mode!r}"
        assert spec.world >= 2, "a rank group has at least two ranks"
        assert not spec.gpus or len(spec.gpus) == spec.world, "one GPU per rank"
        assert spec.tp >= 1 and spec.world % spec.tp == 0, "data-parallel groups of tp ranks"
        assert spec.tp == 1 or spec.distributes, "tp groups apply to the distributing modes"
        spec.store_port = spec.store_port or _free_port()
        spec.pub_port = spec.pub_port or _free_port()
        spec.pull_port = spec.pull_port or _free_port()
        self.spec = spec
        self.procs: list = []
        import zmq

        self._zctx = zmq.Context()
        self.pub = self._zctx.socket(zmq.PUB)
        self.pub.bind(f"tcp://{spec.host}:{spec.pub_port}")
        self.pull = self._zctx.socket(zmq.PULL)
        self.pull.bind(f"tcp://{spec.host}:{spec.pull_port}")
        self.model = self.engine = self.group = None

    def start(self) -> AREngine:
        spec = self.spec
        ctx = mp.get_context("spawn")
        for r in range(1, spec.world):
            p = ctx.Process(target=_follower_main, args=(spec, r), daemon=True, name=f"rank-group-{r}")
            p.start()
            self.procs.append(p)
        device = torch.device("cuda", torch.cuda.current_device()) if spec.gpus else torch.device("cpu")
        self.group, self.model, self.engine = _build_rank(spec, 0, device)
        return self.engine

    def wait_ready(self):
        import zmq

        pending = set(range(1, self.spec.world))
        deadline = time.monotonic() + self.spec.report_timeout_s
        while pending:
            if self.pull.poll(timeout=1000, flags=zmq.POLLIN):
                msg = self.pull.recv_pyobj()
                if "error" in msg:
                    raise RuntimeError(f"rank {msg['error']} of the stage group failed:\n{msg['trace']}")
                pending.discard(msg.get("ready"))
            self.check_alive()
            if time.monotonic() > deadline:
                raise TimeoutError(f"stage group ranks {sorted(pending)} not ready")
        # subscribers that connected late would miss the first message: a short settle pause
        time.sleep(0.2)

    def check_alive(self):
        for i, p in enumerate(self.procs):
            if not p.is_alive():
                raise RuntimeError(f"rank {i + 1} of the stage group exited (code {p.exitcode})")

    def publish(self, msg: dict):
        self.pub.send_pyobj(msg)

    def poll_errors(self):
        """Non-blocking: raises if a follower reported a failure (modes without per-iteration reports)."""
        import zmq

        while self.pull.poll(timeout=0, flags=zmq.POLLIN):
            msg = self.pull.recv_pyobj()
            if "error" in msg:
                raise RuntimeError(f"rank {msg['error']} of the stage group failed:\n{msg['trace']}")

    def reports(self, it: int) -> list[dict]:
        """One report per follower for iteration `it` (bounded wait)."""
        import zmq

        got: dict[int, dict] = {}
        deadline = time.monotonic() + self.spec.report_timeout_s
        while len(got) < self.spec.world - 1:
            if self.pull.poll(timeout=200, flags=zmq.POLLIN):
                msg = self.pull.recv_pyobj()
                if "error" in msg:
                    raise RuntimeError(f"rank {msg['error']} of the stage group failed:\n{msg['trace']}")
                if msg.get("it") == it:
                    got[msg["rank"]] = msg
                continue
            self.check_alive()
            if time.monotonic() > deadline:
                raise TimeoutError(f"stage group: no report for iteration {it}")
        return [got[r] for r in sorted(got)]

    def stop(self):
        try:
            self.publish({"kind": "stop"})
        except Exception:
            pass
        if self.engine is not None:
            # the decode graphs reference the exchange buffers: drop them, then release the
            # buffers together with the followers (a collective over the host group)
            self.engine.runner.graphs.clear()
            if self.engine.runner.is_cuda:
                torch.cuda.synchronize()
            closer = getattr(self.model, "close_parallel", None)
            if closer is not None:
                try:
                    closer()
                except Exception:  # a follower that already died cannot meet the barrier
                    log.exception("closing the stage group's peer buffers")
        for p in self.procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
        self.pub.close(0)
        self.pull.close(0)
        self._zctx.term()


class GroupedAREngine(ThreadedAREngine):
    """The leader's engine thread: the ThreadedAREngine loop plus the group protocol."""

    def __init__(self, engine: AREngine, group: StageRankGroup):
        super().__init__(engine)
        self.rg = group
        self.spec = group.spec
        self._owner: dict[str, int] = {}               # rid -> rank (distributing modes)
        self._remote: dict[str, ARRequest] = {}        # requests served by a follower
        self._load = [0] * self.spec.groups          # requests per data-parallel group
        self._follower_work = [False] * self.spec.world
        self.served_local = 0    # requests this rank ran (distributing modes)
        self.served_remote = 0   # requests a follower ran

    def stop(self):
        super().stop()
        self.rg.stop()

    def _route(self, r: ARRequest, events: list):
        for ev in events:
            if ev[0] == "tok":
                _, rid, tok = ev
                req = self._remote.get(rid)
                if req is not None:
                    req.output_ids.append(tok)
                    if req.first_token_time is None:
                        req.first_token_time = time.perf_counter()
                    if req.on_token is not None:
                        req.on_token(req, tok, {})
            else:
                _, rid, out_ids, reason = ev
                req = self._remote.pop(rid, None)
                owner = self._owner.pop(rid, None)
                if owner is not None:
                    self._load[owner] -= 1
                if req is not None:
                    req.output_ids = list(out_ids)
                    req.finish_reason = reason
                    req.finished = True
                    req.finish_time = time.perf_counter()
                    self._deliver(req)

    def _run(self):
        from ..utils.hostdev import own_stream

        eng = self.engine
        spec = self.spec
        stream = own_stream(eng.runner.device) if eng.runner.is_cuda else None
        if stream is not None:
            torch.cuda.set_stream(stream)
        it = 0
        try:
            eng.runner.capture_all()
            self.rg.wait_ready()
            while True:
                with self._cv:
                    while (not self._inbox and not eng.has_work() and not any(self._follower_work)
                           and not self._stop):
                        self._cv.wait(timeout=0.5)
                    if self._stop:
                        return
                    inbox = list(self._inbox)
                    self._inbox.clear()
                items, local = [], []
                for kind, x in inbox:
                    if kind == "add":
                        if spec.distributes:
                            dst = min(range(spec.groups), key=lambda g: (self._load[g], g))
                            self._load[dst] += 1
                            self._owner[x.rid] = dst
                            if dst == 0:
                                local.append((kind, x))
                                self.served_local += 1
                                if spec.tp > 1:      # the other ranks of the leader's group
                                    items.append(("add", 0, _stable_copy(x)))
                            else:
                                self.served_remote += 1
                                self._remote[x.rid] = x
                                items.append(("add", dst, _stable_copy(x)))
                        else:
                            items.append(("add", -1, _stable_copy(x)))
                            local.append((kind, x))
                    elif kind == "abort":
                        dst = self._owner.get(x, 0) if spec.distributes else -1
                        if dst != 0 or spec.tp > 1:
                            items.append(("abort", dst, x))
                        if dst in (0, -1):
                            local.append((kind, x))
                for kind, x in local:
                    if kind == "add":
                        try:
                            eng.add_request(x)
                        except Exception as exc:
                            x.finished, x.finish_reason = True, f"error: {exc}"
                            self._deliver(x)
                    else:
                        r = eng.requests.get(x)
                        if r is not None and eng.abort(x):
                            self._deliver(r)
                step = eng.has_work() or any(self._follower_work) or any(k == "add" for k, _, _ in items)
                self.rg.publish({"kind": "iter", "it": it, "items": items, "step": step})
                if step:
                    for r in _step(eng, self.rg.model, spec):
                        if spec.distributes:
                            self._owner.pop(r.rid, None)
                            self._load[0] -= 1
                        self._deliver(r)
                if spec.distributes:
                    for rep in self.rg.reports(it):
                        self._follower_work[rep["rank"]] = rep["has_work"]
                        self._route(None, rep["events"])
                else:
                    self.rg.poll_errors()
                    if it % 64 == 0:
                        self.rg.check_alive()
                it += 1
        except BaseException as exc:
            log.exception("rank-group engine loop failed")
            self.error = exc
            for rid, (loop, fut) in list(self._futures.items()):
                loop.call_soon_threadsafe(lambda f=fut, e=exc: f.done() or f.set_exception(e))
            self._futures.clear()
