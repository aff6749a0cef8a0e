"""ZMQ queues carrying msgpack-encoded messages between processes.

PUSH/PULL connect the API server, tokenizer workers and scheduler rank 0;
PUB/SUB fans raw request bytes out from rank 0 to the other TP ranks without
re-encoding (``get_raw`` / ``put_raw``).
"""

from __future__ import annotations

from typing import Callable, Dict, Generic, TypeVar

import msgpack
import zmq
import zmq.asyncio

T = TypeVar("T")


def _open(ctx, kind: int, addr: str, create: bool):
    sock = ctx.socket(kind)
    sock.setsockopt(zmq.LINGER, 0)
    if create:
        sock.bind(addr)
    else:
        sock.connect(addr)
    return sock


class _Base:
    def stop(self) -> None:
        self.socket.close()
        self.context.term()


class ZmqPushQueue(_Base, Generic[T]):
    def __init__(self, addr: str, create: bool, encoder: Callable[[T], Dict]):
        self.context = zmq.Context()
        self.socket = _open(self.context, zmq.PUSH, addr, create)
        self.encoder = encoder

    def put(self, obj: T) -> None:
        self.socket.send(msgpack.packb(self.encoder(obj), use_bin_type=True), copy=False)


class ZmqAsyncPushQueue(_Base, Generic[T]):
    def __init__(self, addr: str, create: bool, encoder: Callable[[T], Dict]):
        self.context = zmq.asyncio.Context()
        self.socket = _open(self.context, zmq.PUSH, addr, create)
        self.encoder = encoder

    async def put(self, obj: T) -> None:
        await self.socket.send(msgpack.packb(self.encoder(obj), use_bin_type=True), copy=False)


class ZmqPullQueue(_Base, Generic[T]):
    def __init__(self, addr: str, create: bool, decoder: Callable[[Dict], T]):
        self.context = zmq.Context()
        self.socket = _open(self.context, zmq.PULL, addr, create)
        self.decoder = decoder

    def get(self) -> T:
        return self.decode(self.socket.recv())

    def get_raw(self) -> bytes:
        return self.socket.recv()

    def decode(self, raw: bytes) -> T:
        return self.decoder(msgpack.unpackb(raw, raw=False))

    def empty(self) -> bool:
        return self.socket.poll(timeout=0) == 0

    def poll(self, timeout_ms: int) -> bool:
        return self.socket.poll(timeout=timeout_ms) != 0


class ZmqAsyncPullQueue(_Base, Generic[T]):
    def __init__(self, addr: str, create: bool, decoder: Callable[[Dict], T]):
        self.context = zmq.asyncio.Context()
        self.socket = _open(self.context, zmq.PULL, addr, create)
        self.decoder = decoder

    async def get(self) -> T:
        return self.decoder(msgpack.unpackb(await self.socket.recv(), raw=False))


class ZmqPubQueue(_Base, Generic[T]):
    def __init__(self, addr: str, create: bool, encoder: Callable[[T], Dict]):
        self.context = zmq.Context()
        self.socket = _open(self.context, zmq.PUB, addr, create)
        self.encoder = encoder

    def put(self, obj: T) -> None:
        self.socket.send(msgpack.packb(self.encoder(obj), use_bin_type=True), copy=False)

    def put_raw(self, raw: bytes) -> None:
        self.socket.send(raw, copy=False)


class ZmqSubQueue(_Base, Generic[T]):
    def __init__(self, addr: str, create: bool, decoder: Callable[[Dict], T]):
        self.context = zmq.Context()
        self.socket = _open(self.context, zmq.SUB, addr, create)
        self.socket.setsockopt_string(zmq.SUBSCRIBE, "")
        self.decoder = decoder

    def get(self) -> T:
        return self.decoder(msgpack.unpackb(self.socket.recv(), raw=False))

    def empty(self) -> bool:
        return self.socket.poll(timeout=0) == 0

    def poll(self, timeout_ms: int) -> bool:
        return self.socket.poll(timeout=timeout_ms) != 0
