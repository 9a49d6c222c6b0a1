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
    def __init__(self, device: str = "cuda", **_):
        self.device = device
        self._keep: dict[str, list[torch.Tensor]] = {}

    async def put_async(self, buffer, request_id):
        buf = buffer.contiguous()
        if not buf.is_cuda:
            buf = buf.to(self.device)
        torch.cuda.current_stream(buf.device).synchronize()
        self._keep.setdefault(request_id, []).append(buf)
        fn, args = reduce_tensor(buf)
        blob = base64.b64encode(pickle.dumps((fn, args))).decode()
        return RelayOperation({"relay": "cuda_ipc", "handle": blob, "nbytes": int(buf.numel() * buf.element_size())})

    async def get_async(self, metadata, dest=None):
        fn, args = pickle.loads(base64.b64decode(metadata["handle"]))
        src = fn(*args)
        out = dest if dest is not None else torch.empty_like(src, device=self.device)
        out.copy_(src)
        return RelayOperation(metadata, result=out)

    def cleanup(self, request_id):
        self._keep.pop(request_id, None)
