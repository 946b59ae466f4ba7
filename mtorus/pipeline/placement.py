"""Topology-aware stage placement and torus hop distance (C++ core).

Reference: crates/mt-pipeline/src/placement.rs -- stage i sits at the torus
coordinates of linear rank i; hop distance sums the wrap-around distance
min(|a-b|, size-|a-b|) per axis.  On one NVSwitch node every GPU pair is one
hop, so the placement only matters across nodes.
"""
from .._ext import host as _host

_C = _host()
topology_aware_placement = _C.topology_aware_placement
compute_hop_distance = _C.compute_hop_distance
torus_distance = _C.torus_distance

__all__ = ["topology_aware_placement", "compute_hop_distance", "torus_distance"]
