"""asyncio adapter of the threaded paged engine to the executor-side engine
contract: ``await generate(rid, ARRequest, on_chunk, stream_fn)`` returns the
finished request; ``on_chunk((token, info))`` fires per generated token on
the event loop; ``abort(rid)``."""
from __future__ import annotations

import asyncio

from .engine import AREngine, ThreadedAREngine
from .request import ARRequest


class PagedAREngineAdapter:
    def __init__(self, engine: AREngine, threaded: ThreadedAREngine | None = None):
        """``threaded``: the engine thread to use (a rank group's leader loop), default a plain one."""
        self.threaded = threaded if threaded is not None else ThreadedAREngine(engine)
        self._started = False

    @property
    def engine(self) -> AREngine:
        return self.threaded.engine

    def start(self):
        if not self._started:
            self.threaded.start()
            self._started = True

    def stop(self):
        if self._started:
            self.threaded.stop()
            self._started = False

    def stats(self) -> dict:
        """Scheduler queues and KV-cache occupancy of the paged engine (read without locking:
        a snapshot for monitoring)."""
        e = self.engine
        pool = e.pool
        used = pool.num_pages - pool.free_pages
        return {"requests_running": len(e.running), "requests_waiting": len(e.waiting),
                "kv_pages_used": used, "kv_pages_total": pool.num_pages,
                "kv_usage": round(used / pool.num_pages, 4) if pool.num_pages else 0.0,
                "steps": getattr(self.threaded, "steps", 0),
                "step_ms": round(getattr(self.threaded, "step_ms_ema", 0.0), 3)}

    async def generate(self, rid: str, req: ARRequest, on_chunk=None, stream_fn=None) -> ARRequest:
        self.start()
        if self.threaded.error is not None:
            raise RuntimeError(f"AR engine failed: {self.threaded.error}")
        req.rid = rid
        fut, q = self.threaded.submit(req, stream=on_chunk is not None)
        if q is not None:
            while True:
                item = await q.get()
                if item is None:
                    break
                on_chunk(item)
        r = await fut
        if r.finish_reason and r.finish_reason.startswith("error"):
            raise RuntimeError(r.finish_reason)
        return r

    def abort(self, rid: str):
        self.threaded.abort(rid)
