"""Communicator interface (C++ core, ``mtorus._C``).

Reference: crates/mt-comm/src/collective.rs -- the ``Communicator`` trait
(send / recv / all_reduce / broadcast / all_gather / rank / world_size) over
byte buffers and ``ReduceOp {Sum, Product, Min, Max, Mean}``.  ``all_reduce``
takes an extra element type (default little-endian u64, the reference Mock's
interpretation).  Errors raise ``CommError`` (``CommTimeout`` for expired
deadlines).

Python subclasses of ``Communicator`` (for example ``NcclCommunicator``) can be
wrapped by the C++ ``TopologyAwareComm``.
"""
from .._ext import host as _host

_C = _host()

Communicator = _C.Communicator
ReduceOp = _C.ReduceOp
DType = _C.DType
CommError = _C.CommError
CommTimeout = _C.CommTimeout
FaultRule = _C.FaultRule
FaultPlan = _C.FaultPlan
reduce_buffers = _C.reduce_buffers


def u64(v: int) -> bytes:
    """Little-endian u64 encoding used by the reference's tests and Mock."""
    return int(v).to_bytes(8, "little")


def from_u64(b: bytes) -> int:
    return int.from_bytes(b[:8], "little")


__all__ = ["Communicator", "ReduceOp", "DType", "CommError", "CommTimeout", "FaultRule", "FaultPlan",
           "reduce_buffers", "u64", "from_u64"]
