"""Parity: crates/mt-core/src/topology/{device,mesh,torus,hybrid,discovery,coordinator}.rs tests."""
import pytest

from mtorus.core.coordinator import CollectiveOp, DummyCommunicator
from mtorus.core.topology import (DiscoveryConfig, GPUDevice, IntraNodeMesh, MeshTorusHybrid, TorusCoordinates,
                                  TorusDimensions, discover_devices, discover_manual, discover_mesh)

TC, TD = TorusCoordinates, TorusDimensions


# ---------------------------------------------------------------- device.rs
def test_device_new():
    d = GPUDevice(0, 1, "0000:01:00.0", [1, 2, 3])
    assert (d.id, d.numa_node, d.pci_bus_id, d.nvlink_peers) == (0, 1, "0000:01:00.0", [1, 2, 3])


def test_device_simple():
    d = GPUDevice.simple(2, 4)
    assert d.id == 2 and d.nvlink_peers == [0, 1, 3] and d.numa_node is None
    assert d.pci_bus_id == "0000:02:00.0"


@pytest.mark.parametrize("id_,peer,expected", [(0, 1, True), (0, 3, True), (0, 4, False)])
def test_is_nvlink_peer(id_, peer, expected):
    assert GPUDevice(id_, None, "0000:00:00.0", [1, 2, 3]).is_nvlink_peer(peer) == expected


def test_peer_count():
    assert GPUDevice(0, None, "0000:00:00.0", [1, 2, 3]).peer_count() == 3


# ---------------------------------------------------------------- mesh.rs
@pytest.mark.parametrize("n", [4, 8, 1])
def test_full_mesh(n):
    m = IntraNodeMesh.full_mesh(n)
    assert m.device_count() == n and m.all_pairs_nvlinked()


def test_empty_mesh_fails():
    with pytest.raises(ValueError):
        IntraNodeMesh.full_mesh(0)


def test_custom_mesh():
    m = IntraNodeMesh([GPUDevice(0, 0, "0000:01:00.0", [1, 2]), GPUDevice(1, 0, "0000:02:00.0", [0, 2]),
                       GPUDevice(2, 1, "0000:03:00.0", [0, 1])])
    assert m.device_count() == 3 and m.are_nvlinked(0, 1) and m.are_nvlinked(1, 2) and m.are_nvlinked(0, 2)


def test_device_lookup():
    d = IntraNodeMesh.full_mesh(4).device(2)
    assert d.id == 2 and d.nvlink_peers == [0, 1, 3]


def test_device_not_found():
    assert IntraNodeMesh.full_mesh(2).device(5) is None


def test_invalid_device_id_fails():
    with pytest.raises(ValueError):
        IntraNodeMesh([GPUDevice(0, None, "0000:00:00.0", [1]), GPUDevice(5, None, "0000:01:00.0", [0])])


# ---------------------------------------------------------------- torus.rs
def test_2d_coordinates():
    c = TC.new_2d(1, 2)
    assert (c.x, c.y, c.z, c.is_3d()) == (1, 2, None, False)


def test_3d_coordinates():
    c = TC.new_3d(1, 2, 3)
    assert (c.x, c.y, c.z, c.is_3d()) == (1, 2, 3, True)


def test_linear_index_and_back():
    assert TC.new_2d(2, 1).linear_index(TD.new_2d(4, 3)) == 6
    assert TC.new_3d(2, 1, 1).linear_index(TD.new_3d(4, 3, 2)) == 18
    assert TC.from_linear(6, TD.new_2d(4, 3)) == TC.new_2d(2, 1)
    assert TC.from_linear(18, TD.new_3d(4, 3, 2)) == TC.new_3d(2, 1, 1)


def test_2d_neighbors_interior():
    nb = [c for c, _ in TC.new_2d(1, 1).neighbors(TD.new_2d(4, 4))]
    assert len(nb) == 4
    for c in (TC.new_2d(2, 1), TC.new_2d(0, 1), TC.new_2d(1, 2), TC.new_2d(1, 0)):
        assert c in nb


def test_neighbor_order_and_axes():
    nb = TC.new_2d(1, 1).neighbors(TD.new_2d(4, 4))
    assert [a for _, a in nb] == [0, 0, 1, 1]
    assert nb[0][0] == TC.new_2d(2, 1) and nb[1][0] == TC.new_2d(0, 1)


def test_2d_neighbors_wrap():
    d, c = TD.new_2d(3, 3), TC.new_2d(0, 0)
    assert c.neighbor(d, 0, True) == TC.new_2d(1, 0)
    assert c.neighbor(d, 0, False) == TC.new_2d(2, 0)
    assert c.neighbor(d, 1, True) == TC.new_2d(0, 1)
    assert c.neighbor(d, 1, False) == TC.new_2d(0, 2)


def test_3d_neighbors():
    nb = [c for c, _ in TC.new_3d(1, 1, 1).neighbors(TD.new_3d(3, 3, 3))]
    assert len(nb) == 6
    for c in (TC.new_3d(2, 1, 1), TC.new_3d(0, 1, 1), TC.new_3d(1, 2, 1), TC.new_3d(1, 0, 1), TC.new_3d(1, 1, 2),
              TC.new_3d(1, 1, 0)):
        assert c in nb


def test_3d_neighbors_wrap():
    d, c = TD.new_3d(3, 3, 3), TC.new_3d(0, 0, 0)
    assert c.neighbor(d, 0, False) == TC.new_3d(2, 0, 0)
    assert c.neighbor(d, 1, False) == TC.new_3d(0, 2, 0)
    assert c.neighbor(d, 2, False) == TC.new_3d(0, 0, 2)
    assert c.neighbor(d, 2, True) == TC.new_3d(0, 0, 1)


def test_axis_out_of_range_raises():
    with pytest.raises(IndexError):
        TC.new_2d(0, 0).neighbor(TD.new_2d(2, 2), 3, True)


def test_axis2_on_2d_coords_gives_z():
    assert TC.new_2d(0, 0).neighbor(TD.new_2d(2, 2), 2, True).z == 0


def test_dimensions():
    assert TD.new_2d(4, 3).total_nodes() == 12
    assert TD.new_3d(4, 3, 2).total_nodes() == 24
    assert TD.new_2d(4, 3).axis_count() == 2 and TD.new_3d(4, 3, 2).axis_count() == 3


# ---------------------------------------------------------------- hybrid.rs
def test_2d_hybrid():
    h = MeshTorusHybrid.new_2d(3, 3, 4)
    assert (h.total_nodes(), h.devices_per_node(), h.total_devices()) == (9, 4, 36)


def test_3d_hybrid():
    h = MeshTorusHybrid.new_3d(2, 2, 2, 8)
    assert (h.total_nodes(), h.devices_per_node(), h.total_devices()) == (8, 8, 64)


@pytest.mark.parametrize("args", [(0, 3, 4), (3, 0, 4), (3, 3, 0)])
def test_2d_zero_fails(args):
    with pytest.raises(ValueError):
        MeshTorusHybrid.new_2d(*args)


@pytest.mark.parametrize("args", [(0, 2, 2, 4), (2, 0, 2, 4), (2, 2, 0, 4), (2, 2, 2, 0)])
def test_3d_zero_fails(args):
    with pytest.raises(ValueError):
        MeshTorusHybrid.new_3d(*args)


def test_node_at():
    assert MeshTorusHybrid.new_2d(3, 3, 4).node_at(TC.new_2d(1, 2)).device_count() == 4
    assert MeshTorusHybrid.new_3d(2, 3, 2, 4).node_at(TC.new_3d(1, 2, 1)).device_count() == 4


def test_global_device_id():
    h = MeshTorusHybrid.new_2d(3, 3, 4)
    assert h.global_device_id(TC.new_2d(1, 1), 0) == 16 and h.global_device_id(TC.new_2d(1, 1), 3) == 19


def test_node_neighbors():
    h = MeshTorusHybrid.new_2d(3, 3, 4)
    nb = [c for c, _ in h.node_neighbors(TC.new_2d(1, 1))]
    assert len(nb) == 4 and TC.new_2d(2, 1) in nb and TC.new_2d(1, 0) in nb
    assert len(MeshTorusHybrid.new_3d(3, 3, 3, 4).node_neighbors(TC.new_3d(1, 1, 1))) == 6
    corner = [c for c, _ in MeshTorusHybrid.new_2d(3, 3, 2).node_neighbors(TC.new_2d(0, 0))]
    assert len(corner) == 4 and TC.new_2d(2, 0) in corner and TC.new_2d(0, 2) in corner


@pytest.mark.parametrize("h", [MeshTorusHybrid.new_2d(4, 3, 2), MeshTorusHybrid.new_3d(3, 4, 2, 2)])
def test_rank_roundtrip(h):
    for r in range(h.total_nodes()):
        assert h.node_rank(h.rank_to_coords(r)) == r


def test_hybrid_equality():
    assert MeshTorusHybrid.new_2d(2, 2, 2) == MeshTorusHybrid.new_2d(2, 2, 2)
    assert MeshTorusHybrid.new_2d(2, 2, 2) != MeshTorusHybrid.new_2d(2, 2, 4)


# ---------------------------------------------------------------- discovery.rs
def test_manual_discovery_default():
    d = discover_manual(DiscoveryConfig())
    assert len(d) == 8 and d[0].id == 0 and d[7].id == 7
    assert d[0].pci_bus_id == "0000:01:00.0" and d[7].pci_bus_id == "0000:08:00.0"


def test_manual_discovery_custom_count():
    d = discover_manual(DiscoveryConfig(num_devices_override=4))
    assert len(d) == 4 and d[0].nvlink_peers == [1, 2, 3]


def test_discover_mesh():
    m = discover_mesh(DiscoveryConfig(assume_full_mesh=True, num_devices_override=4))
    assert m.device_count() == 4 and m.all_pairs_nvlinked()
    assert discover_mesh(DiscoveryConfig(assume_full_mesh=False, num_devices_override=3)).device_count() == 3


def test_discover_devices_override():
    assert len(discover_devices(DiscoveryConfig(num_devices_override=2))) == 2


def test_default_config():
    c = DiscoveryConfig()
    assert c.assume_full_mesh and c.num_devices_override is None


def test_numa_assignment():
    d = discover_manual(DiscoveryConfig(num_devices_override=8))
    assert [d[i].numa_node for i in (0, 3, 4, 7)] == [0, 0, 1, 1]


# ---------------------------------------------------------------- coordinator.rs
def test_collective_op_display():
    assert [o.to_string() for o in (CollectiveOp.AllReduce, CollectiveOp.Broadcast, CollectiveOp.AllGather,
                             CollectiveOp.ReduceScatter)] == ["AllReduce", "Broadcast", "AllGather", "ReduceScatter"]
    assert CollectiveOp.AllReduce == CollectiveOp.AllReduce and CollectiveOp.AllReduce != CollectiveOp.Broadcast


def test_dummy_communicator():
    c = DummyCommunicator(0, 4)
    data = bytes([1, 2, 3, 4])
    r = c.nearest_neighbor_exchange(data, 0)
    assert len(r) == 4 and r[0] == data
    assert c.all_reduce_mesh(data, [0, 1, 2, 3]) == data
    assert c.pipeline_stage_sendrecv(data, 1) == data
    assert c.route_collective(CollectiveOp.AllReduce, data) == data
    for op in (CollectiveOp.AllReduce, CollectiveOp.Broadcast, CollectiveOp.AllGather, CollectiveOp.ReduceScatter):
        assert DummyCommunicator(0, 2).route_collective(op, b"\x2a") == b"\x2a"
    assert len(DummyCommunicator(0, 2).nearest_neighbor_exchange(b"\x01", 0)) == 2


def test_numa_binding_from_sysfs(tmp_path):
    """NUMA-aware host affinity: the GPU's PCI device -> its NUMA node -> that node's
    CPUs, read from a stand-in sysfs tree (nothing is applied in the test)."""
    import os

    from mtorus.core.topology import bind_to_gpu_numa, numa_cpus, parse_cpulist

    assert parse_cpulist("0-3,8,10-11\n") == [0, 1, 2, 3, 8, 10, 11]
    allowed = sorted(os.sched_getaffinity(0))
    node = tmp_path / "devices/system/node/node1"
    node.mkdir(parents=True)
    (node / "cpulist").write_text(f"{allowed[0]}-{allowed[-1]}\n")
    dev = tmp_path / "bus/pci/devices/0000:1b:00.0"
    dev.mkdir(parents=True)
    (dev / "numa_node").write_text("1\n")
    assert numa_cpus(1, str(tmp_path)) == list(range(allowed[0], allowed[-1] + 1))
    got = bind_to_gpu_numa(bus_id="0000:1B:00.0", sysfs=str(tmp_path), apply=False)
    assert got == allowed  # intersected with what the process may use
    (dev / "numa_node").write_text("-1\n")  # no NUMA information: no binding
    assert bind_to_gpu_numa(bus_id="0000:1b:00.0", sysfs=str(tmp_path), apply=False) is None
    assert bind_to_gpu_numa(bus_id="0000:99:00.0", sysfs=str(tmp_path), apply=False) is None
