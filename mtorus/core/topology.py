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


def _numa_of(bus_id: str, sysfs: str = "/sys") -> Optional[int]:
    path = f"{sysfs}/bus/pci/devices/{bus_id.lower()}/numa_node"
    try:
        with open(path) as f:
            v = int(f.read().strip())
        return v if v >= 0 else None
    except (OSError, ValueError):
        return None


def parse_cpulist(text: str) -> List[int]:
    """Linux cpulist syntax ("0-15,32-47,64") -> sorted CPU ids."""
    cpus = set()
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            lo, hi = part.split("-")
            cpus.update(range(int(lo), int(hi) + 1))
        else:
            cpus.add(int(part))
    return sorted(cpus)


def numa_cpus(node: int, sysfs: str = "/sys") -> List[int]:
    """CPUs of NUMA node ``node`` (empty when sysfs does not list them)."""
    try:
        with open(f"{sysfs}/devices/system/node/node{node}/cpulist") as f:
            return parse_cpulist(f.read())
    except (OSError, ValueError):
        return []


def _cuda_bus_id(index: int) -> Optional[str]:
    import torch

    if not torch.cuda.is_available() or index >= torch.cuda.device_count():
        return None
    props = torch.cuda.get_device_properties(index)
    bus = getattr(props, "pci_bus_id", None)
    if isinstance(bus, int):
        bus = f"{getattr(props, 'pci_domain_id', 0):04x}:{bus:02x}:{getattr(props, 'pci_device_id', 0):02x}.0"
    return bus


def bind_to_gpu_numa(device_index: int = 0, bus_id: Optional[str] = None, sysfs: str = "/sys",
                     apply: bool = True) -> Optional[List[int]]:
    """Pin this process's host threads to the CPUs of the NUMA node the GPU hangs off
    (host-to-device copies, the data loader and kernel launches then stay on the
    socket next to the GPU).  On Linux an affinity belongs to a thread, so the set is
    applied to every thread the process has now (``/proc/self/task``: CUDA driver and
    torch pool threads started before this call included); threads created later
    inherit it from their creator.  Only CPU affinity changes; nothing on the GPU is
    touched.  The CPU set is intersected with the CPUs the process may use now.
    Returns the CPUs bound to, or None when the node, its CPU list or the
    intersection is unknown or empty (then nothing changes)."""
    import os

    bus = bus_id or _cuda_bus_id(device_index)
    node = _numa_of(bus, sysfs) if bus else None
    if node is None:
        return None
    cpus = set(numa_cpus(node, sysfs))
    allowed = set(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else cpus
    cpus &= allowed
    if not cpus:
        return None
    if apply and hasattr(os, "sched_setaffinity"):
        tids = []
        try:
            tids = [int(t) for t in os.listdir("/proc/self/task")]
        except OSError:
            pass
        for tid in tids:
            try:
                os.sched_setaffinity(tid, cpus)
            except OSError:  # the thread exited meanwhile
                pass
        os.sched_setaffinity(0, cpus)
    return sorted(cpus)


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
    "topology_aware_placement", "compute_hop_distance", "torus_distance", "parse_cpulist", "numa_cpus",
    "bind_to_gpu_numa",
]
