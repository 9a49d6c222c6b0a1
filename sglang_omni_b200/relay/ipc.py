"""Same-node GPU relay through CUDA IPC: the sender exports the device buffer
(torch's CUDA IPC handle reduction) and keeps it alive until the request is
cleaned up; the receiver maps it and copies into its own memory.  Used for
stage hand-offs between processes on GPUs of one node without a host
round-trip (the reference's same-GPU streaming path,
sglang_omni/pipeline/worker/runtime.py:539-641)."""
from __future__ import annotations

import base64
import pickle

import torch
from torch.multiprocessing.reductions import reduce_tensor

from .base import Relay, RelayOperation, register_relay


@register_relay("cuda_ipc")
class CudaIpcRelay(Relay):
    """Sender: no host synchronisation per put.  The producer's stream records an
    interprocess CUDA event (from a pool whose IPC handles are exported once), the
    receiver's stream waits on that event before its copy.  Buffers stay referenced
    until the request is cleaned up (torch's IPC reference counting keeps the memory
    alive while the receiver maps it); the receiver caches opened events by handle."""

    def __init__(self, device: str = "cuda", **_):
        self.device = device
        self._keep: dict[str, list] = {}
        self._free_events: list = []          # (event, handle) pairs not referenced by a live request
        self._opened: dict[bytes, torch.cuda.Event] = {}

    def _event(self):
        if self._free_events:
            return self._free_events.pop()
        ev = torch.cuda.Event(interprocess=True)
        return ev, None

    async def put_async(self, buffer, request_id):
        buf = buffer.contiguous()
        if not buf.is_cuda:
            buf = buf.to(self.device, non_blocking=True)
        ev, handle = self._event()
        ev.record(torch.cuda.current_stream(buf.device))
        if handle is None:
            handle = ev.ipc_handle()
        self._keep.setdefault(request_id, []).append((buf, ev, handle))
        fn, args = reduce_tensor(buf)
        blob = base64.b64encode(pickle.dumps((fn, args))).decode()
        return RelayOperation({"relay": "cuda_ipc", "handle": blob, "event": base64.b64encode(handle).decode(),
                               "device": buf.device.index, "nbytes": int(buf.numel() * buf.element_size())})

    async def get_async(self, metadata, dest=None):
        fn, args = pickle.loads(base64.b64decode(metadata["handle"]))
        src = fn(*args)
        eh = base64.b64decode(metadata["event"])
        ev = self._opened.get(eh)
        if ev is None:
            ev = torch.cuda.Event.from_ipc_handle(src.device, eh)
            self._opened[eh] = ev
        stream = torch.cuda.current_stream(src.device)
        stream.wait_event(ev)                 # the producer's data is ready on the device
        out = dest if dest is not None else torch.empty_like(src, device=self.device)
        out.copy_(src, non_blocking=True)
        return RelayOperation(metadata, result=out)

    def cleanup(self, request_id):
        for _buf, ev, handle in self._keep.pop(request_id, []):
            self._free_events.append((ev, handle))
