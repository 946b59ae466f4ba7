"""TCP communicator (C++ sockets) and frame helpers.

Reference: crates/mt-comm/src/tcp.rs.  Frame = u64 little-endian length +
payload.  ``TcpCommunicator(rank, addresses)`` binds ``addresses[rank]``,
accepts lower ranks, dials higher ranks (retrying until ``connect_timeout_s``)
and implements every Communicator method, collectives as ring algorithms.
``send_frame`` / ``recv_frame`` work on any connected Python socket;
``async_send_frame`` / ``async_recv_frame`` on asyncio streams.
"""
from __future__ import annotations

import asyncio
import socket
import struct
from typing import List, Optional

from .._ext import host as _host

_C = _host()
TcpCommunicator = _C.TcpCommunicator
LEN_PREFIX_SIZE = 8


def send_frame(sock: socket.socket, data: bytes) -> None:
    _C.tcp_send_frame(sock.fileno(), bytes(data))


def recv_frame(sock: socket.socket, timeout_s: float = 30.0) -> bytes:
    return _C.tcp_recv_frame(sock.fileno(), float(timeout_s))


async def async_send_frame(writer: asyncio.StreamWriter, data: bytes) -> None:
    writer.write(struct.pack("<Q", len(data)) + bytes(data))
    await writer.drain()


async def async_recv_frame(reader: asyncio.StreamReader) -> bytes:
    (n,) = struct.unpack("<Q", await reader.readexactly(LEN_PREFIX_SIZE))
    return await reader.readexactly(n) if n else b""


def free_ports(n: int, host: str = "127.0.0.1") -> List[int]:
    socks, ports = [], []
    for _ in range(n):
        s = socket.socket()
        s.bind((host, 0))
        socks.append(s)
        ports.append(s.getsockname()[1])
    for s in socks:
        s.close()
    return ports


def tcp_world_from_store(store, rank: int, world_size: int, host: str = "127.0.0.1",
                         connect_timeout_s: float = 30.0, op_timeout_s: float = 60.0) -> "TcpCommunicator":
    """Bring up a TCP world across processes: each rank binds an ephemeral port,
    publishes it in a key-value store (e.g. torch.distributed.TCPStore), then
    lower ranks dial higher ranks."""
    comm = TcpCommunicator(rank, [f"{host}:0" if r == rank else f"{host}:1" for r in range(world_size)],
                           0.05, op_timeout_s, False)
    store.set(f"mtorus_tcp_{rank}", f"{host}:{comm.port()}")
    addrs = [store.get(f"mtorus_tcp_{r}").decode() for r in range(world_size)]
    for dst in range(rank + 1, world_size):
        comm.connect_to(dst, addrs[dst], connect_timeout_s)
    missing = comm.wait_connected(connect_timeout_s)
    if missing:
        raise _C.CommError(f"rank {rank}: peers {missing} never connected")
    return comm


__all__ = ["TcpCommunicator", "send_frame", "recv_frame", "async_send_frame", "async_recv_frame",
           "free_ports", "tcp_world_from_store", "LEN_PREFIX_SIZE"]
