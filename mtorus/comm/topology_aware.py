"""Topology-aware communicator (C++ ``TopologyAwareComm``).

Reference: crates/mt-comm/src/topology_aware.rs.  The inner communicator's rank
is a torus node rank.  ``exchange_with_neighbors`` sends to and receives from
every +/- neighbour on each axis, ``perform_collective`` maps CollectiveOp onto
the inner communicator (ReduceScatter = all-reduce + slice), ``reduce_on_mesh``
ignores its group like the reference (``reduce_on_group`` honours it), and the
``TopologyAwareCommunicator`` methods fall back to the caller's data on errors.

Over the device backend (``mtorus.comm.device.SymmCommunicator``) the inner
communicator implements ``exchange``, and ``exchange_with_neighbors`` /
``nearest_neighbor_exchange`` move the whole exchange in one peer-memory kernel
(every neighbour's message pulled over NVLink at once) instead of a send and a
receive per neighbour.  For device tensors, ``SymmCommunicator.
exchange_neighbors_tensor`` stores straight into each neighbour's receive slot
(``halo_kernel``).
"""
from .._ext import host as _host

TopologyAwareComm = _host().TopologyAwareComm

__all__ = ["TopologyAwareComm"]
