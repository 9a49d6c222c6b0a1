"""Payload <-> relay adapter.

``write_payload`` walks the payload's data (dicts / lists / tuples), lifts
every tensor out (replacing it with a placeholder), and ships the tensors
through the stage's relay: the in-process relay passes the tensor objects
themselves; byte relays get ONE flat uint8 buffer (all tensors packed back to
back, 16-byte aligned) so a hand-off is a single transfer.  The tensor-free
skeleton rides in the control message.  Stream chunks use the same path
(``write_blob`` / ``read_blob``).

Reference counterpart: sglang_omni/pipeline/worker/data_plane.py:16-244.
"""
from __future__ import annotations

import pickle
from typing import Any

import torch

from ...proto import OmniRequest, StagePayload
from ...relay import Relay

_ALIGN = 16


def _extract(obj: Any, out: list[torch.Tensor]):
    if isinstance(obj, torch.Tensor):
        out.append(obj)
        return {"__tensor__": len(out) - 1}
    if isinstance(obj, dict):
        return {k: _extract(v, out) for k, v in obj.items()}
    if isinstance(obj, list):
        return [_extract(v, out) for v in obj]
    if isinstance(obj, tuple):
        return {"__tuple__": [_extract(v, out) for v in obj]}
    return obj


def _restore(obj: Any, tensors: list[torch.Tensor]):
    if isinstance(obj, dict):
        if "__tensor__" in obj and len(obj) == 1:
            return tensors[obj["__tensor__"]]
        if "__tuple__" in obj and len(obj) == 1:
            return tuple(_restore(v, tensors) for v in obj["__tuple__"])
        return {k: _restore(v, tensors) for k, v in obj.items()}
    if isinstance(obj, list):
        return [_restore(v, tensors) for v in obj]
    return obj


class DataPlaneAdapter:
    def __init__(self, relay: Relay, device: str | torch.device = "cpu"):
        self.relay = relay
        self.device = torch.device(device)

    @property
    def zero_copy(self) -> bool:
        return getattr(self.relay, "relay_type", "") == "inproc"

    async def _ship(self, request_id: str, skeleton: Any, tensors: list[torch.Tensor], dst: int | None):
        if not tensors:
            return {"skeleton": pickle.dumps(skeleton), "tensors": None}
        if self.zero_copy:
            handles = []
            for t in tensors:
                op = await self.relay.put_async(t, request_id)
                handles.append(op.metadata)
            return {"skeleton": pickle.dumps(skeleton), "tensors": {"mode": "objects", "handles": handles}}
        info, offs, total = [], [], 0
        for t in tensors:
            nbytes = t.numel() * t.element_size()
            offs.append(total)
            info.append((str(t.dtype).replace("torch.", ""), list(t.shape), total, nbytes))
            total += (nbytes + _ALIGN - 1) // _ALIGN * _ALIGN
        dev = tensors[0].device if all(t.device == tensors[0].device for t in tensors) else torch.device("cpu")
        flat = torch.empty(max(total, 1), dtype=torch.uint8, device=dev)
        for t, o in zip(tensors, offs):
            n = t.numel() * t.element_size()
            if n:
                flat[o:o + n].copy_(t.detach().contiguous().view(torch.uint8).reshape(-1).to(dev), non_blocking=True)
        kwargs = {"dst": dst} if dst is not None and self.relay.relay_type == "nccl" else {}
        op = await self.relay.put_async(flat, request_id, **kwargs)
        return {"skeleton": pickle.dumps(skeleton), "tensors": {"mode": "flat", "relay": op.metadata, "info": info}}

    async def _unship(self, meta: dict[str, Any]):
        skeleton = pickle.loads(meta["skeleton"])
        tm = meta.get("tensors")
        if tm is None:
            return skeleton
        tensors = []
        if tm["mode"] == "objects":
            for h in tm["handles"]:
                op = await self.relay.get_async(h)
                tensors.append(await op.wait_for_completion())
        else:
            op = await self.relay.get_async(tm["relay"])
            flat = await op.wait_for_completion()
            for dtype, shape, off, nbytes in tm["info"]:
                dt = getattr(torch, dtype)
                seg = flat[off:off + nbytes].clone() if nbytes else torch.empty(0, dtype=torch.uint8,
                                                                               device=flat.device)
                tensors.append(seg.view(dt).reshape(shape))
        return _restore(skeleton, tensors)

    async def write_payload(self, request_id: str, payload: StagePayload, dst: int | None = None) -> dict:
        tensors: list[torch.Tensor] = []
        skel = {"request_id": payload.request_id, "request": _extract(payload.request.to_dict(), tensors),
                "data": _extract(payload.data, tensors)}
        return await self._ship(request_id, skel, tensors, dst)

    async def read_payload(self, metadata: dict) -> StagePayload:
        d = await self._unship(metadata)
        return StagePayload(request_id=d["request_id"], request=OmniRequest.from_dict(d["request"]), data=d["data"])

    async def write_blob(self, request_id: str, obj: Any, dst: int | None = None) -> dict:
        tensors: list[torch.Tensor] = []
        skel = _extract(obj, tensors)
        return await self._ship(request_id, skel, tensors, dst)

    async def read_blob(self, metadata: dict) -> Any:
        return await self._unship(metadata)
