"""ZMQ control plane (asyncio).

Topology (same as sglang_omni/pipeline/control_plane.py:59-443):
  * each stage binds one PULL socket for work / data-ready / stream-chunk
    messages and lazily connects PUSH sockets to the stages it sends to;
  * stages PUSH completions and stream chunks to the coordinator's PULL;
  * the coordinator PUBlishes aborts, every stage SUBscribes.
Messages are msgpack dicts (see proto.messages); tensors never travel here.

Endpoints ``local://...`` (single-process pipelines) skip ZMQ and msgpack: a
PUSH/PULL pair is one asyncio queue of message objects and PUB/SUB a list of
queues, all owned by the process's event loop.  Per-token stream chunks
between stages and to the coordinator then cost one queue operation each.
"""
from __future__ import annotations

import asyncio
import logging
from typing import Any

import msgpack
import zmq
import zmq.asyncio

from ..proto import parse_message

log = logging.getLogger(__name__)


def serialize_message(msg) -> bytes:
    return msgpack.packb(msg.to_dict(), use_bin_type=True)


def deserialize_message(data: bytes):
    return parse_message(msgpack.unpackb(data, raw=False))


class ControlPlaneContext:
    _ctx: zmq.asyncio.Context | None = None

    @classmethod
    def get(cls) -> zmq.asyncio.Context:
        if cls._ctx is None or cls._ctx.closed:
            cls._ctx = zmq.asyncio.Context.instance()
        return cls._ctx


LOCAL_PREFIX = "local://"
_LOCAL_QUEUES: dict[str, asyncio.Queue] = {}
_LOCAL_SUBS: dict[str, list[asyncio.Queue]] = {}


def _local_queue(endpoint: str) -> asyncio.Queue:
    q = _LOCAL_QUEUES.get(endpoint)
    if q is None:
        q = _LOCAL_QUEUES[endpoint] = asyncio.Queue()
    return q


class _LocalPush:
    def __init__(self, endpoint: str):
        self.endpoint = endpoint

    async def send(self, msg) -> None:
        _local_queue(self.endpoint).put_nowait(msg)

    def close(self):
        pass


class _LocalPull:
    def __init__(self, endpoint: str):
        self.endpoint = endpoint
        _LOCAL_QUEUES[endpoint] = _LOCAL_QUEUES.get(endpoint) or asyncio.Queue()

    async def recv(self):
        return await _local_queue(self.endpoint).get()

    def close(self):
        _LOCAL_QUEUES.pop(self.endpoint, None)


class _LocalPub:
    def __init__(self, endpoint: str):
        self.endpoint = endpoint
        _LOCAL_SUBS.setdefault(endpoint, [])

    async def publish(self, msg) -> None:
        for q in _LOCAL_SUBS.get(self.endpoint, []):
            q.put_nowait(msg)

    def close(self):
        _LOCAL_SUBS.pop(self.endpoint, None)


class _LocalSub:
    def __init__(self, endpoint: str):
        self.endpoint = endpoint
        self.q: asyncio.Queue = asyncio.Queue()
        _LOCAL_SUBS.setdefault(endpoint, []).append(self.q)

    async def recv(self):
        return await self.q.get()

    def close(self):
        subs = _LOCAL_SUBS.get(self.endpoint)
        if subs and self.q in subs:
            subs.remove(self.q)


def _push(endpoint: str, bind: bool = False):
    sock = _LocalPush(endpoint) if endpoint.startswith(LOCAL_PREFIX) else PushSocket(endpoint, bind)
    from . import faults

    return faults.FaultyPush(sock, endpoint) if faults.active() else sock


def _pull(endpoint: str):
    return _LocalPull(endpoint) if endpoint.startswith(LOCAL_PREFIX) else PullSocket(endpoint, bind=True)


def _pub(endpoint: str):
    return _LocalPub(endpoint) if endpoint.startswith(LOCAL_PREFIX) else PubSocket(endpoint)


def _sub(endpoint: str):
    return _LocalSub(endpoint) if endpoint.startswith(LOCAL_PREFIX) else SubSocket(endpoint)


class _Sock:
    def __init__(self, endpoint: str, kind: int, bind: bool):
        self.endpoint = endpoint
        self.sock = ControlPlaneContext.get().socket(kind)
        self.sock.setsockopt(zmq.LINGER, 0)
        if bind:
            self.sock.bind(endpoint)
        else:
            self.sock.connect(endpoint)

    def close(self):
        try:
            self.sock.close(linger=0)
        except Exception:  # pragma: no cover
            pass


class PushSocket(_Sock):
    def __init__(self, endpoint: str, bind: bool = False):
        super().__init__(endpoint, zmq.PUSH, bind)

    async def send(self, msg) -> None:
        await self.sock.send(serialize_message(msg))


class PullSocket(_Sock):
    def __init__(self, endpoint: str, bind: bool = True):
        super().__init__(endpoint, zmq.PULL, bind)

    async def recv(self):
        return deserialize_message(await self.sock.recv())


class PubSocket(_Sock):
    def __init__(self, endpoint: str):
        super().__init__(endpoint, zmq.PUB, True)

    async def publish(self, msg) -> None:
        await self.sock.send(serialize_message(msg))


class SubSocket(_Sock):
    def __init__(self, endpoint: str):
        super().__init__(endpoint, zmq.SUB, False)
        self.sock.setsockopt(zmq.SUBSCRIBE, b"")

    async def recv(self):
        return deserialize_message(await self.sock.recv())


class StageControlPlane:
    def __init__(self, stage_name: str, recv_endpoint: str, coordinator_endpoint: str, abort_endpoint: str):
        self.stage_name = stage_name
        self.recv_endpoint = recv_endpoint
        self.coordinator_endpoint = coordinator_endpoint
        self.abort_endpoint = abort_endpoint
        self._pull: PullSocket | None = None
        self._to_coord: PushSocket | None = None
        self._sub: SubSocket | None = None
        self._peers: dict[str, PushSocket] = {}

    def start(self):
        self._pull = _pull(self.recv_endpoint)
        self._to_coord = _push(self.coordinator_endpoint)
        self._sub = _sub(self.abort_endpoint)

    async def recv(self):
        return await self._pull.recv()

    async def recv_abort(self):
        return await self._sub.recv()

    async def send_to_stage(self, endpoint: str, msg) -> None:
        s = self._peers.get(endpoint)
        if s is None:
            s = self._peers[endpoint] = _push(endpoint)
        await s.send(msg)

    async def send_to_coordinator(self, msg) -> None:
        await self._to_coord.send(msg)

    def close(self):
        for s in [self._pull, self._to_coord, self._sub, *self._peers.values()]:
            if s is not None:
                s.close()
        self._peers.clear()


class CoordinatorControlPlane:
    def __init__(self, completion_endpoint: str, abort_endpoint: str):
        self.completion_endpoint = completion_endpoint
        self.abort_endpoint = abort_endpoint
        self._pull: PullSocket | None = None
        self._pub: PubSocket | None = None
        self._stages: dict[str, PushSocket] = {}

    async def start(self):
        self._pull = _pull(self.completion_endpoint)
        self._pub = _pub(self.abort_endpoint)
        await asyncio.sleep(0.05)  # let subscribers connect before the first publish

    async def send_to_stage(self, endpoint: str, msg) -> None:
        s = self._stages.get(endpoint)
        if s is None:
            s = self._stages[endpoint] = _push(endpoint)
        await s.send(msg)

    async def recv(self):
        return await self._pull.recv()

    async def broadcast(self, msg) -> None:
        await self._pub.publish(msg)

    def close(self):
        for s in [self._pull, self._pub, *self._stages.values()]:
            if s is not None:
                s.close()
        self._stages.clear()
