"""Topology-level communication contract.

Reference: crates/mt-core/src/topology/coordinator.rs:3-56 -- ``CollectiveOp``,
the ``TopologyAwareCommunicator`` trait (nearest-neighbour exchange, mesh
all-reduce, pipeline send/recv, collective routing) and ``DummyCommunicator``.
"""
from __future__ import annotations

import abc
from typing import List, Sequence

from .._ext import host as _host

CollectiveOp = _host().CollectiveOp


class TopologyAwareCommunicator(abc.ABC):
    @abc.abstractmethod
    def nearest_neighbor_exchange(self, data: bytes, axis: int) -> List[bytes]: ...

    @abc.abstractmethod
    def all_reduce_mesh(self, data: bytes, group: Sequence[int]) -> bytes: ...

    @abc.abstractmethod
    def pipeline_stage_sendrecv(self, data: bytes, stage_rank: int) -> bytes: ...

    @abc.abstractmethod
    def route_collective(self, op, data: bytes) -> bytes: ...


TopologyAwareCommunicator.register(_host().TopologyAwareComm)


class DummyCommunicator(TopologyAwareCommunicator):
    """Echoes its input; the neighbour exchange returns min(world, 4) copies."""

    def __init__(self, rank: int, world_size: int):
        self.rank = rank
        self.world_size = world_size

    def nearest_neighbor_exchange(self, data: bytes, axis: int) -> List[bytes]:
        return [bytes(data)] * min(self.world_size, 4)

    def all_reduce_mesh(self, data: bytes, group: Sequence[int]) -> bytes:
        return bytes(data)

    def pipeline_stage_sendrecv(self, data: bytes, stage_rank: int) -> bytes:
        return bytes(data)

    def route_collective(self, op, data: bytes) -> bytes:
        return bytes(data)


__all__ = ["CollectiveOp", "TopologyAwareCommunicator", "DummyCommunicator"]
