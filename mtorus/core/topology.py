"""Mesh-torus topology model (C++ core, ``mtorus._C``).

Reference: crates/mt-core/src/topology/{device,mesh,torus,hybrid,discovery}.rs.

* ``GPUDevice``         id, NUMA node, PCI bus id, NVLink peer list (device.rs:1-35)
* ``IntraNodeMesh``     the NVLink mesh inside one node (mesh.rs:3-63)
* ``TorusCoordinates`` / ``TorusDimensions``  2-D/3-D torus math with wrap (torus.rs)
* ``MeshTorusHybrid``   a torus of nodes, each an NVLink full mesh (hybrid.rs)
* ``discover_devices`` / ``discover_mesh``  device discovery (discovery.rs)

On a B200 HGX box the eight GPUs hang off NVSwitch, so every pair is one switch
hop apart: the node mesh is physical, the torus a virtual overlay.  Discovery
queries CUDA for the device count, PCI bus ids and peer-access matrix and reads
each GPU's NUMA node from sysfs; without a GPU (or with an explicit device
count) it reproduces the reference's manual enumeration.
"""
from __future__ import annotations

import os
from typing import List, Optional

from .._ext import host as _host

_C = _host()

GPUDevice = _C.GPUDevice
IntraNodeMesh = _C.IntraNodeMesh
TorusCoordinates = _C.TorusCoordinates
TorusDimensions = _C.TorusDimensions
MeshTorusHybrid = _C.MeshTorusHybrid
DiscoveryConfig = _C.DiscoveryConfig
topology_aware_placement = _C.topology_aware_placement
compute_hop_distance = _C.compute_hop_distance
torus_distance = _C.torus_distance


def discover_manual(config: Optional[DiscoveryConfig] = None) -> List[GPUDevice]:
    """Reference manual enumeration: count = override or 8, NUMA = id / max(count/2, 1),
    bus id ``0000:{id+1:02x}:00.0``, full peer lists (discovery.rs:73-87)."""
    return _C.discover_manual(config or DiscoveryConfig())


def _numa_of(bus_id: str) -> Optional[int]:
    path = f"/sys/bus/pci/devices/{bus_id.lower()}/numa_node"
    try:
        with open(path) as f:
            v = int(f.read().strip())
        return v if v >= 0 else None
    except (OSError, ValueError):
        return None


def discover_cuda(config: Optional[DiscoveryConfig] = None) -> List[GPUDevice]:
    """Query CUDA: device count, PCI bus ids, the real peer-access matrix, NUMA nodes."""
    import torch

    cfg = config or DiscoveryConfig()
    n = torch.cuda.device_count()
    if cfg.num_devices_override is not None:
        n = min(n, cfg.num_devices_override)
    devs = []
    for i in range(n):
        props = torch.cuda.get_device_properties(i)
        bus = getattr(props, "pci_bus_id", None)
        if isinstance(bus, int):
            dom = getattr(props, "pci_domain_id", 0)
            dev = getattr(props, "pci_device_id", 0)
            bus = f"{dom:04x}:{bus:02x}:{dev:02x}.0"
        bus = bus or f"0000:{i + 1:02x}:00.0"
        peers = [j for j in range(n) if j != i and torch.cuda.can_device_access_peer(i, j)]
        devs.append(GPUDevice(i, _numa_of(bus), bus, peers))
    return devs


def discover_devices(config: Optional[DiscoveryConfig] = None) -> List[GPUDevice]:
    """CUDA discovery when GPUs are visible and no count override is given,
    otherwise the reference's manual enumeration (discovery.rs:18-27)."""
    cfg = config or DiscoveryConfig()
    if cfg.num_devices_override is None and not os.environ.get("MTORUS_MANUAL_DISCOVERY"):
        try:
            import torch

            if torch.cuda.is_available() and torch.cuda.device_count() > 0:
                return discover_cuda(cfg)
        except Exception:
            pass
    return discover_manual(cfg)


def discover_mesh(config: Optional[DiscoveryConfig] = None) -> IntraNodeMesh:
    """Node mesh from discovery; peers forced to a full mesh when
    ``assume_full_mesh`` (discovery.rs:29-44)."""
    cfg = config or DiscoveryConfig()
    return _C.mesh_from_devices(discover_devices(cfg), cfg.assume_full_mesh)


__all__ = [
    "GPUDevice", "IntraNodeMesh", "TorusCoordinates", "TorusDimensions", "MeshTorusHybrid",
    "DiscoveryConfig", "discover_devices", "discover_mesh", "discover_manual", "discover_cuda",
    "topology_aware_placement", "compute_hop_distance", "torus_distance",
]
