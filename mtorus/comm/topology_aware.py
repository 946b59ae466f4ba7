"""Topology-aware communicator (C++ ``TopologyAwareComm``).

Reference: crates/mt-comm/src/topology_aware.rs.  The inner communicator's rank
is a torus node rank.  ``exchange_with_neighbors`` sends to and receives from
every +/- neighbour on each axis, ``perform_collective`` maps CollectiveOp onto
the inner communicator (ReduceScatter = all-reduce + slice), ``reduce_on_mesh``
ignores its group like the reference (``reduce_on_group`` honours it), and the
``TopologyAwareCommunicator`` methods fall back to the caller's data on errors.

The device counterpart of the neighbour exchange (direct NVLink peer stores
between GPUs) is ``mtorus.parallel.symm.HaloExchange``.
"""
from .._ext import host as _host

TopologyAwareComm = _host().TopologyAwareComm

__all__ = ["TopologyAwareComm"]
