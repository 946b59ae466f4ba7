"""In-process point-to-point channels.

Reference: crates/mt-comm/src/p2p.rs.  ``P2PChannel.isend`` writes the shared
[src][dst] slot and returns a completed handle; ``irecv`` snapshots the slot at
call time (reference semantics).  ``P2PHandle.wait`` is bounded here
(``timeout_s``; the reference spins forever).  ``AsyncP2PChannel`` is the
asyncio counterpart of the reference's tokio channel.
"""
from __future__ import annotations

import asyncio
from typing import List, Tuple

from .._ext import host as _host

_C = _host()
P2PChannel = _C.P2PChannel
P2PHandle = _C.P2PHandle


class AsyncP2PChannel:
    def __init__(self, rank: int, world_size: int, _shared=None):
        self._rank = rank
        self._world = world_size
        self._buf = _shared if _shared is not None else [[b""] * world_size for _ in range(world_size)]
        self._lock = asyncio.Lock() if _shared is None else None

    @staticmethod
    def create_group(world_size: int) -> List["AsyncP2PChannel"]:
        shared = [[b""] * world_size for _ in range(world_size)]
        chans = [AsyncP2PChannel(r, world_size, shared) for r in range(world_size)]
        lock = asyncio.Lock()
        for c in chans:
            c._lock = lock
        return chans

    async def isend(self, data: bytes, dst: int) -> P2PHandle:
        async with self._lock:
            self._buf[self._rank][dst] = bytes(data)
        h = P2PHandle()
        h.set_result(bytes(data))
        return h

    async def irecv(self, src: int) -> P2PHandle:
        async with self._lock:
            data = self._buf[src][self._rank]
        h = P2PHandle()
        h.set_result(data)
        return h

    async def sendrecv(self, data: bytes, dst: int, src: int) -> Tuple[P2PHandle, P2PHandle]:
        s = await self.isend(data, dst)
        r = await self.irecv(src)
        return s, r

    def rank(self) -> int:
        return self._rank

    def world_size(self) -> int:
        return self._world


__all__ = ["P2PChannel", "P2PHandle", "AsyncP2PChannel"]
