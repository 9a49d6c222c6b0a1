"""Paged autoregressive engine: continuous batching, chunked prefill, KV
retraction, overlap scheduling (the host plans and launches step N+1 before
it reads step N's tokens), CUDA-graph decode.

With ``prefix_cache=True`` finished requests leave their full KV pages in a
page-granular radix tree (``KVPool.enable_prefix_cache``); a later request
whose token prompt starts with the same pages skips their prefill.  Only
requests whose KV is a function of their token ids alone take part (no
embedding overrides, multimodal rows, deep-stack inputs, shifted M-RoPE
positions or captured prompt hidden states); ``extra["prefix_key"]`` puts a
request into a namespace of its own (e.g. one per LoRA or speaker) and
``extra["no_prefix_cache"]`` opts it out.

``AREngine.step()`` is the synchronous core used by benchmarks and tests;
``ThreadedAREngine`` runs the same loop on a dedicated thread and exposes the
engine contract used by the pipeline executors (add_request / stream /
get_result / abort, awaitable from asyncio).

Reference counterparts: OmniEngine normal / overlap step loop
(sglang_omni/engines/omni/engine.py:152-400), SGLangBatchPlanner prefill-first
selection and post-step filtering (sglang_omni/engines/omni/runtime/sglang_ar.py:40-300),
PrefillManager / DecodeManager retraction
(sglang_omni/engines/ar/sglang_backend/scheduler/prefill.py:13-80,
sglang_omni/engines/ar/sglang_backend/scheduler/decode.py:14-78), radix tree
cache (sglang_omni/engines/ar/sglang_backend/scheduler/cache.py:9-30).
"""
from __future__ import annotations

import asyncio
import logging
import threading
import time
from collections import deque

import numpy as np
import torch

from ...utils.hostdev import own_stream
from .kv_pool import PAGE, KVPool
from .request import ARRequest
from .runner import ARModelRunner

log = logging.getLogger(__name__)


class AREngine:
    def __init__(self, model, pool: KVPool, max_batch: int = 64, max_prefill_tokens: int = 8192,
                 max_context: int = 8192, use_graphs: bool = True, overlap: bool = True, eos_token_ids=(),
                 suppress=(-1, -1, -1), track_seen: bool = False, max_slots: int | None = None,
                 prefix_cache: bool = False):
        self.pool = pool
        self.prefix_cache = pool.enable_prefix_cache() if prefix_cache else pool.prefix_cache
        self.max_batch = max_batch
        self.max_prefill_tokens = max_prefill_tokens
        self.max_context = max_context
        self.overlap = overlap
        self.eos_token_ids = tuple(eos_token_ids)
        self.runner = ARModelRunner(model, pool, max_batch=max_batch, max_slots=max_slots or max(256, 2 * max_batch + 2),
                                    max_context=max_context, max_prefill_tokens=max_prefill_tokens,
                                    use_graphs=use_graphs, suppress=suppress, track_seen=track_seen)
        self.waiting: deque[ARRequest] = deque()
        self.prefilling: list[ARRequest] = []
        self.running: list[ARRequest] = []
        self.requests: dict[str, ARRequest] = {}
        self.pending = None
        self._finished_buf: list[ARRequest] = []
        self.num_steps = 0
        self.num_retractions = 0
        self.num_prefix_hit_tokens = 0
        self.last_launched = False

    # ------------------------------------------------------------------ API
    def add_request(self, req: ARRequest):
        if not req.eos_token_ids:
            req.eos_token_ids = self.eos_token_ids
        if len(req.prompt_ids) + req.max_new_tokens > self.max_context:
            raise ValueError(f"request {req.rid}: prompt {req.prompt_len} + {req.max_new_tokens} new tokens "
                             f"exceeds max_context {self.max_context}")
        self.requests[req.rid] = req
        self.waiting.append(req)

    def abort(self, rid: str) -> bool:
        r = self.requests.get(rid)
        if r is None or r.finished:
            return False
        r.aborted = True
        r.finish_reason = "abort"
        self._finish(r)
        return True

    def has_work(self) -> bool:
        return bool(self.waiting or self.prefilling or self.running or self.pending)

    # ------------------------------------------------------------------ prefix cache
    @staticmethod
    def _cacheable(r: ARRequest) -> bool:
        if (r.input_embeds is not None or r.mm_index is not None or r.deepstack is not None
                or r.capture_prompt_layer is not None or r.extra.get("no_prefix_cache")):
            return False
        if r.mrope_positions is not None:  # text-only layouts have plain positions and no delta
            n = r.mrope_positions.shape[1]
            return r.mrope_delta == 0 and n > 0 and int(r.mrope_positions[0, n - 1]) == n - 1
        return True

    @staticmethod
    def _namespace(r: ARRequest) -> int:
        key = r.extra.get("prefix_key")
        return 0 if key is None else hash(key) & 0xFFFFFFFFFFFFFFFF

    def _match_prefix(self, r: ARRequest):
        """Reuses the cached full pages at the start of r's prompt; at least the
        last prompt token is always recomputed (its logits start the decode)."""
        max_blocks = (r.prompt_len - 1) // PAGE
        if max_blocks <= 0:
            return
        seq = np.asarray(r.prefill_ids(0, max_blocks * PAGE), dtype=np.int32)
        nodes, pages = self.prefix_cache.match(self._namespace(r), seq, max_blocks)
        if nodes:
            r.prefix_nodes = list(nodes)
            r.pages = list(pages)
            r.num_cached = len(pages) * PAGE
            r.cached_tokens = max(r.cached_tokens, r.num_cached)
            self.num_prefix_hit_tokens += r.num_cached

    def _release_kv(self, r: ARRequest, keep: bool):
        """Returns r's pages: with ``keep`` its full pages join the prefix cache
        (their KV is final: every position < num_cached has been written, in
        stream order before any later reader), the rest go back to the pool."""
        pc = self.prefix_cache
        if pc is None:
            self.pool.free(r.pages)
        elif keep and self._cacheable(r):
            seq_len = min(r.num_cached, len(r.prompt_ids) + len(r.output_ids))
            nblk = min(seq_len // PAGE, len(r.pages))
            seq = np.asarray((list(r.prompt_ids) + list(r.output_ids))[:nblk * PAGE], dtype=np.int32)
            dup = pc.insert_release(self._namespace(r), seq, list(r.pages[:nblk]), r.prefix_nodes)
            self.pool.free(list(dup) + list(r.pages[nblk:]))
        else:
            pc.release(r.prefix_nodes)
            self.pool.free(r.pages[len(r.prefix_nodes):])
        r.pages = []
        r.prefix_nodes = []

    # ------------------------------------------------------------------ scheduling
    def _tokens_in_flight(self, r: ARRequest) -> int:
        return r.folded + (1 if r.prefill_done else 0) + r.scheduled_decodes

    def _schedule_prefill(self):
        budget = self.max_prefill_tokens
        chunks = []
        cands = list(self.prefilling) + list(self.waiting)
        active = len(self.running) + len(self.prefilling)
        for r in cands:
            if r.finished:
                continue
            new = r.slot < 0
            if new and active >= self.max_batch:
                break
            if new and self.prefix_cache is not None and r.num_cached == 0 and not r.pages and self._cacheable(r):
                self._match_prefix(r)
            remaining = r.prompt_len - r.num_cached
            n = min(remaining, budget)
            if n <= 0:
                continue
            need = KVPool.pages_for(r.num_cached + n) - len(r.pages)
            # keep one page of headroom per running request for its next decode token
            if not self.pool.can_alloc(need + (1 if new else 0)):
                break
            if need > 0:
                r.pages.extend(self.pool.alloc(need))
            if new:
                self.runner.assign_slot(r)
                self.waiting.remove(r)
                self.prefilling.append(r)
                active += 1
            chunks.append((r, r.num_cached, r.num_cached + n))
            r.num_cached += n
            budget -= n
            if r.prefill_done:
                self.prefilling.remove(r)
                self.running.append(r)
            if budget <= 0:
                break
        return chunks

    def _drain(self):
        """Reads the in-flight step so host state is exact (needed before a retraction)."""
        if self.pending is not None:
            self._finished_buf.extend(self._process(self.pending))
            self.pending = None

    def _retract_one(self) -> bool:
        self._drain()
        if len(self.running) <= 1:
            return False
        victim = max(self.running, key=lambda r: r.arrival)
        self.running.remove(victim)
        self._release_kv(victim, keep=True)  # its re-prefill can match its own pages if they survive
        # recompute later: the generated tokens are re-prefilled after the prompt
        victim.folded = len(victim.output_ids)
        victim.num_cached = 0
        victim.scheduled_decodes = 0
        self.runner.release_slot(victim)
        self.waiting.appendleft(victim)
        self.num_retractions += 1
        return True

    def _schedule_decode(self):
        batch = [r for r in self.running
                 if not r.finished and self._tokens_in_flight(r) < r.max_new_tokens][: self.max_batch]
        while batch:
            need = sum(1 for r in batch if r.num_cached % 64 == 0 and r.num_cached // 64 >= len(r.pages))
            if self.pool.ensure_free(need):  # the decode metadata builder allocates from the free list
                break
            if not self._retract_one():
                raise RuntimeError("KV pool exhausted and nothing to retract")
            batch = [r for r in batch if r in self.running]
        return batch

    # ------------------------------------------------------------------ step
    def step(self) -> list[ARRequest]:
        """One engine iteration; returns requests that finished during it."""
        launched = None
        chunks = self._schedule_prefill()
        if chunks:
            launched = self.runner.prefill(chunks)
        else:
            batch = self._schedule_decode()
            if batch:
                launched = self.runner.decode(batch)
        finished, self._finished_buf = self._finished_buf, []
        if self.overlap:
            if self.pending is not None:
                finished += self._process(self.pending)
            self.pending = launched
        elif launched is not None:
            finished += self._process(launched)
        if launched is None and self.pending is not None:
            finished += self._process(self.pending)
            self.pending = None
        self.num_steps += 1
        self.last_launched = launched is not None   # one model forward ran in this step
        return finished

    def _process(self, out) -> list[ARRequest]:
        if out is None:
            return []
        if out["event"] is not None:
            out["event"].synchronize()
        toks = out["host"].tolist()
        now = time.perf_counter()
        finished = []
        captured = out.get("captured") or {}
        for i, (r, t) in enumerate(zip(out["reqs"], toks)):
            if r.finished:
                continue
            r.output_ids.append(int(t))
            if r.first_token_time is None:
                r.first_token_time = now
            if r.on_token is not None:
                info = {k: v[i] for k, v in captured.items() if isinstance(k, int)}
                info["hidden"] = out["hidden"][i]
                r.on_token(r, int(t), info)
            if r.check_stop(int(t)):
                self._finish(r)
                finished.append(r)
        return finished

    def _finish(self, r: ARRequest):
        if r.finished:
            return
        r.finished = True
        r.finish_time = time.perf_counter()
        for lst in (self.running, self.prefilling):
            if r in lst:
                lst.remove(r)
        if r in self.waiting:
            self.waiting.remove(r)
        self._release_kv(r, keep=not r.aborted)
        self.runner.release_slot(r)

    def run_until_idle(self, max_steps: int = 10_000_000) -> None:
        n = 0
        while self.has_work() and n < max_steps:
            self.step()
            n += 1

    def generate(self, reqs: list[ARRequest]) -> list[ARRequest]:
        for r in reqs:
            self.add_request(r)
        self.run_until_idle()
        return reqs


class ThreadedAREngine:
    """Runs an AREngine step loop on its own thread; results are delivered to
    asyncio futures / queues of the loop that submitted the request."""

    def __init__(self, engine: AREngine):
        self.engine = engine
        self.steps = 0            # engine steps run by this thread
        self.step_ms_ema = 0.0    # host time of a step (moving average over ~10 steps)
        self._cv = threading.Condition()
        self._inbox: deque = deque()
        self._stop = False
        self._thread = threading.Thread(target=self._run, name="ar-engine", daemon=True)
        self._futures: dict[str, tuple[asyncio.AbstractEventLoop, asyncio.Future]] = {}
        self._queues: dict[str, tuple[asyncio.AbstractEventLoop, asyncio.Queue]] = {}
        self.error: BaseException | None = None

    def start(self):
        self._thread.start()
        return self

    def stop(self):
        with self._cv:
            self._stop = True
            self._cv.notify_all()
        self._thread.join(timeout=30)

    def submit(self, req: ARRequest, stream: bool = False):
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        self._futures[req.rid] = (loop, fut)
        q = None
        if stream:
            q = asyncio.Queue()
            self._queues[req.rid] = (loop, q)
        user_cb = req.on_token

        def on_token(r, tok, info, _q=q, _loop=loop, _cb=user_cb):
            if _cb is not None:
                _cb(r, tok, info)
            if _q is not None:
                _loop.call_soon_threadsafe(_q.put_nowait, (tok, info))

        req.on_token = on_token
        with self._cv:
            self._inbox.append(("add", req))
            self._cv.notify_all()
        return fut, q

    def abort(self, rid: str):
        with self._cv:
            self._inbox.append(("abort", rid))
            self._cv.notify_all()

    def _deliver(self, r: ARRequest):
        item = self._futures.pop(r.rid, None)
        if item is not None:
            loop, fut = item
            loop.call_soon_threadsafe(lambda: fut.done() or fut.set_result(r))
        q = self._queues.pop(r.rid, None)
        if q is not None:
            loop, qq = q
            loop.call_soon_threadsafe(qq.put_nowait, None)

    def _run(self):
        eng = self.engine
        stream = own_stream(eng.runner.device) if eng.runner.is_cuda else None
        if stream is not None:
            torch.cuda.set_stream(stream)  # this thread's work queues behind nobody else's
        try:
            eng.runner.capture_all()  # every decode bucket, before the first request (not on its latency path)
            while True:
                with self._cv:
                    while not self._inbox and not eng.has_work() and not self._stop:
                        self._cv.wait(timeout=0.5)
                    if self._stop:
                        return
                    inbox = list(self._inbox)
                    self._inbox.clear()
                for kind, x in inbox:
                    if kind == "add":
                        try:
                            eng.add_request(x)
                        except Exception as exc:  # reject this request only
                            x.finished, x.finish_reason = True, f"error: {exc}"
                            self._deliver(x)
                    elif kind == "abort":
                        r = eng.requests.get(x)
                        if r is not None and eng.abort(x):
                            self._deliver(r)
                if eng.has_work():
                    t0 = time.perf_counter()
                    done = eng.step()
                    ms = (time.perf_counter() - t0) * 1e3
                    self.steps += 1
                    self.step_ms_ema = ms if self.steps == 1 else 0.9 * self.step_ms_ema + 0.1 * ms
                    for r in done:
                        self._deliver(r)
        except BaseException as exc:  # engine failure fails every in-flight request
            log.exception("AR engine loop failed")
            self.error = exc
            for rid, (loop, fut) in list(self._futures.items()):
                loop.call_soon_threadsafe(lambda f=fut, e=exc: f.done() or f.set_exception(e))
            self._futures.clear()
