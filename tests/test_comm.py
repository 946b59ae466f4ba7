"""Parity: crates/mt-comm/src/{collective,mock,p2p,tcp,topology_aware}.rs tests, plus real
multi-rank semantics of the in-process, TCP and torch.distributed (gloo) backends and
host-side fault injection."""
import asyncio
import socket
import struct
import threading

import pytest

from mtorus.comm import (AsyncP2PChannel, CommError, CommTimeout, DType, FaultPlan, FaultRule, MockCommunicator,
                         P2PChannel, P2PHandle, ReduceOp, TcpCommunicator, TopologyAwareComm, from_u64, local_world,
                         recv_frame, run_threads, send_frame, u64)
from mtorus.comm.tcp import async_recv_frame, async_send_frame, free_ports
from mtorus.core.coordinator import CollectiveOp
from mtorus.core.topology import MeshTorusHybrid, TorusCoordinates


# ---------------------------------------------------------------- collective.rs
@pytest.mark.parametrize("op,name", [(ReduceOp.Sum, "Sum"), (ReduceOp.Product, "Product"), (ReduceOp.Min, "Min"),
                                     (ReduceOp.Max, "Max"), (ReduceOp.Mean, "Mean")])
def test_reduce_op_display(op, name):
    assert op.to_string() == name


def test_reduce_op_equality():
    assert ReduceOp.Sum == ReduceOp.Sum and ReduceOp.Sum != ReduceOp.Max


# ---------------------------------------------------------------- mock.rs
def test_mock_all_reduce_sum():
    assert from_u64(MockCommunicator.create_world(4)[0].all_reduce(u64(10), ReduceOp.Sum)) == 40


def test_mock_all_reduce_sum_multi_element():
    r = MockCommunicator.create_world(4)[0].all_reduce(u64(1) + u64(2) + u64(3), ReduceOp.Sum)
    assert len(r) == 24 and [from_u64(r[i:i + 8]) for i in (0, 8, 16)] == [4, 8, 12]


@pytest.mark.parametrize("n,op,x,expected", [(3, ReduceOp.Product, 3, 27), (4, ReduceOp.Min, 10, 10),
                                             (4, ReduceOp.Max, 10, 10), (4, ReduceOp.Mean, 10, 10)])
def test_mock_all_reduce_ops(n, op, x, expected):
    assert from_u64(MockCommunicator.create_world(n)[0].all_reduce(u64(x), op)) == expected


def test_mock_broadcast_send_recv_gather():
    comms = MockCommunicator.create_world(4)
    for c in comms:
        assert c.broadcast(bytes([42, 43, 44]), 0) == bytes([42, 43, 44])
    c2 = MockCommunicator.create_world(2)
    c2[0].send(bytes([1, 2, 3, 4]), 1)
    assert c2[1].recv(0) == bytes([1, 2, 3, 4])
    r = MockCommunicator.create_world(3)[0].all_gather(bytes([99]))
    assert len(r) == 3 and all(x == bytes([99]) for x in r)
    assert comms[0].rank() == 0 and comms[3].rank() == 3 and comms[0].world_size() == 4


def test_mock_recv_is_non_blocking_and_non_consuming():
    c = MockCommunicator.create_world(2)
    assert c[1].recv(0) == b""
    c[0].send(b"a", 1)
    c[0].send(b"b", 1)  # last write wins
    assert c[1].recv(0) == b"b" and c[1].recv(0) == b"b"


def test_mock_invalid_ranks():
    c = MockCommunicator.create_world(2)
    with pytest.raises(CommError):
        c[0].send(b"\x01", 5)
    with pytest.raises(CommError):
        c[0].recv(5)
    with pytest.raises(CommError):
        c[0].broadcast(b"\x01", 5)


# ---------------------------------------------------------------- p2p.rs
def test_p2p_isend_irecv_and_sendrecv():
    ch = P2PChannel.create_group(2)
    ch[0].isend(bytes([1, 2, 3, 4]), 1)
    assert ch[1].irecv(0).wait() == bytes([1, 2, 3, 4])
    ch[0].isend(bytes([10, 20]), 1)
    ch[1].isend(bytes([30, 40]), 0)
    assert ch[0].irecv(1).wait() == bytes([30, 40]) and ch[1].irecv(0).wait() == bytes([10, 20])
    ch4 = P2PChannel.create_group(4)
    ch4[0].isend(bytes([42]), 2)
    assert ch4[2].irecv(0).wait() == bytes([42])
    assert ch4[0].rank() == 0 and ch4[3].rank() == 3 and ch4[0].world_size() == 4
    s, r = ch[0].sendrecv(b"x", 1, 1)
    assert s.wait() == b"x" and r.wait() == bytes([30, 40])


def test_p2p_handle_try_get_and_bounded_wait():
    h = P2PHandle()
    assert h.try_get() is None
    with pytest.raises(CommTimeout):
        h.wait(0.05)
    h.set_result(bytes([1, 2, 3]))
    assert h.try_get() == bytes([1, 2, 3])


def test_async_p2p():
    async def main():
        ch = AsyncP2PChannel.create_group(2)
        await ch[0].isend(bytes([5, 6, 7, 8]), 1)
        assert (await ch[1].irecv(0)).wait() == bytes([5, 6, 7, 8])
        await ch[0].isend(bytes([100]), 1)
        await ch[1].isend(bytes([200]), 0)
        assert (await ch[0].irecv(1)).wait() == bytes([200])
        assert (await ch[1].irecv(0)).wait() == bytes([100])
        c4 = AsyncP2PChannel.create_group(4)
        assert c4[0].rank() == 0 and c4[0].world_size() == 4

    asyncio.run(main())


# ---------------------------------------------------------------- tcp.rs (frames)
def _echo_server(transform, n):
    srv = socket.socket()
    srv.bind(("127.0.0.1", 0))
    srv.listen(1)
    port = srv.getsockname()[1]

    def run():
        conn, _ = srv.accept()
        for _ in range(n):
            send_frame(conn, transform(recv_frame(conn, 10.0)))
        conn.close()
        srv.close()

    t = threading.Thread(target=run, daemon=True)
    t.start()
    return port, t


@pytest.mark.parametrize("msg", [b"hello world", bytes(i % 256 for i in range(65536)), b""])
def test_tcp_roundtrip(msg):
    port, t = _echo_server(lambda d: d, 1)
    c = socket.create_connection(("127.0.0.1", port))
    send_frame(c, msg)
    assert recv_frame(c, 10.0) == msg
    c.close()
    t.join(5)


def test_tcp_multiple_messages():
    port, t = _echo_server(lambda d: bytes((b + 1) % 256 for b in d), 5)
    c = socket.create_connection(("127.0.0.1", port))
    for i in range(5):
        send_frame(c, bytes([i] * 10))
        assert recv_frame(c, 10.0) == bytes([(i + 1) % 256] * 10)
    c.close()
    t.join(5)


def test_tcp_frame_format_is_u64_le_length_prefix():
    a, b = socket.socketpair()
    send_frame(a, b"abc")
    raw = b.recv(11)
    assert raw == struct.pack("<Q", 3) + b"abc"


def test_tcp_async_frames():
    async def main():
        got = []

        async def handle(r, w):
            got.append(await async_recv_frame(r))
            await async_send_frame(w, got[-1])
            w.close()

        srv = await asyncio.start_server(handle, "127.0.0.1", 0)
        port = srv.sockets[0].getsockname()[1]
        r, w = await asyncio.open_connection("127.0.0.1", port)
        await async_send_frame(w, b"ping")
        assert await async_recv_frame(r) == b"ping"
        w.close()
        srv.close()

    asyncio.run(main())


def test_tcp_communicator_rank_with_unreachable_peers():
    comm = TcpCommunicator(2, ["127.0.0.1:0"] * 3, connect_timeout_s=0.1)
    assert comm.rank() == 2 and comm.world_size() == 3
    with pytest.raises(CommError):
        comm.send(b"x", 0)
    comm.close()


def _tcp_world(n):
    ports = free_ports(n)
    addrs = [f"127.0.0.1:{p}" for p in ports]
    comms = [None] * n

    def mk(r):
        comms[r] = TcpCommunicator(r, addrs, connect_timeout_s=10.0, op_timeout_s=20.0)

    ts = [threading.Thread(target=mk, args=(r,)) for r in range(n)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(30)
    for c in comms:
        assert c.wait_connected(10.0) == []
    return comms


def test_tcp_communicator_collectives():
    comms = _tcp_world(4)
    try:
        res = run_threads(comms, lambda c: c.all_reduce(u64(c.rank() + 1) + u64(10 * (c.rank() + 1)), ReduceOp.Sum))
        assert all(from_u64(r[:8]) == 10 and from_u64(r[8:]) == 100 for r in res)
        import numpy as np

        res = run_threads(comms, lambda c: c.all_reduce(np.arange(1003, dtype=np.float32).tobytes() if c.rank() == 0
                                                        else np.ones(1003, dtype=np.float32).tobytes(),
                                                        ReduceOp.Max, DType.F32))
        exp = np.maximum(np.arange(1003, dtype=np.float32), 1).tobytes()
        assert all(r == exp for r in res)
        res = run_threads(comms, lambda c: c.broadcast(b"root-data" if c.rank() == 2 else b"", 2))
        assert all(r == b"root-data" for r in res)
        res = run_threads(comms, lambda c: c.all_gather(bytes([c.rank()] * (c.rank() + 1))))
        assert all(r == [bytes([k] * (k + 1)) for k in range(4)] for r in res)
        res = run_threads(comms, lambda c: c.all_reduce(u64(8 * (c.rank() + 1)), ReduceOp.Mean))
        assert all(from_u64(r) == 20 for r in res)
    finally:
        for c in comms:
            c.close()


def test_tcp_concurrent_send_and_recv_do_not_deadlock():
    comms = _tcp_world(2)
    big = bytes(4 * 1024 * 1024)

    def body(c):
        peer = 1 - c.rank()
        t = threading.Thread(target=c.send, args=(big, peer))
        t.start()
        got = c.recv(peer)
        t.join()
        return len(got)

    assert run_threads(comms, body) == [len(big), len(big)]
    for c in comms:
        c.close()


def test_tcp_fault_plan_drop_yields_timeout():
    ports = free_ports(2)
    addrs = [f"127.0.0.1:{p}" for p in ports]
    comms = [None, None]

    def mk(r):
        comms[r] = TcpCommunicator(r, addrs, connect_timeout_s=10.0, op_timeout_s=0.5)

    ts = [threading.Thread(target=mk, args=(r,)) for r in range(2)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(30)
    assert comms[1].wait_connected(10.0) == []
    plan = FaultPlan()
    plan.add(FaultRule(rank=0, at_op=0, op_kind="send", action=FaultRule.Action.Drop))
    comms[0].set_fault_plan(plan)
    comms[0].send(b"lost", 1)        # dropped on the host before it reaches the socket
    with pytest.raises(CommTimeout):
        comms[1].recv(0)             # the receiver's deadline ends the wait
    comms[0].send(b"next", 1)
    assert comms[1].recv(0) == b"next"
    for c in comms:
        c.close()


# ---------------------------------------------------------------- topology_aware.rs
def _torus(w, h):
    topo = MeshTorusHybrid.new_2d(w, h, 2)
    return [TopologyAwareComm(m, topo) for m in MockCommunicator.create_world(w * h)]


def test_topology_aware_rank_and_coords():
    c = _torus(3, 3)
    assert c[0].rank() == 0 and c[8].rank() == 8 and c[0].world_size() == 9
    assert c[0].rank_coords() == TorusCoordinates.new_2d(0, 0) and c[5].rank_coords() == TorusCoordinates.new_2d(2, 1)


def test_exchange_with_neighbors():
    c = _torus(3, 3)
    assert len(c[4].exchange_with_neighbors(bytes([42]))) == 4
    r = c[0].exchange_with_neighbors(bytes([99]))
    ranks = [x for x, _ in r]
    assert len(r) == 4 and 1 in ranks and 3 in ranks


def test_perform_collectives():
    c = _torus(2, 2)
    assert from_u64(c[0].perform_collective(CollectiveOp.AllReduce, u64(10))) == 40
    assert c[1].perform_collective(CollectiveOp.Broadcast, bytes([1, 2, 3])) == bytes([1, 2, 3])
    assert len(c[0].perform_collective(CollectiveOp.AllGather, bytes([42]))) == 4
    assert len(c[0].perform_collective(CollectiveOp.ReduceScatter, u64(10))) == 8 // 4


def test_trait_methods():
    c = _torus(3, 3)
    assert len(c[4].nearest_neighbor_exchange(bytes([1, 2, 3]), 0)) == 2
    c = _torus(2, 2)
    assert from_u64(c[0].all_reduce_mesh(u64(42), [0, 1, 2, 3])) == 168
    c[1].inner().send(u64(99), 0)
    assert from_u64(c[0].pipeline_stage_sendrecv(u64(99), 1)) == 99
    assert c[0].route_collective(CollectiveOp.Broadcast, bytes([42])) == bytes([42])
    assert from_u64(c[0].reduce_on_mesh(u64(5), [0, 1])) == 20


def test_3d_topology_and_accessors():
    topo = MeshTorusHybrid.new_3d(2, 2, 2, 2)
    comms = [TopologyAwareComm(m, topo) for m in MockCommunicator.create_world(8)]
    assert len(comms) == 8 and comms[0].world_size() == 8
    assert comms[7].rank_coords() == TorusCoordinates.new_3d(1, 1, 1)
    c = _torus(3, 3)
    assert c[0].inner().rank() == 0 and c[0].topology().total_nodes() == 9


# ---------------------------------------------------------------- real semantics (LocalWorld)
def test_local_world_collectives_and_p2p():
    w = local_world(4, 10.0)
    res = run_threads(w, lambda c: from_u64(c.all_reduce(u64(c.rank() + 1), ReduceOp.Sum)))
    assert res == [10, 10, 10, 10]
    res = run_threads(w, lambda c: from_u64(c.all_reduce(u64(c.rank() + 1), ReduceOp.Product)))
    assert res == [24] * 4
    res = run_threads(w, lambda c: c.broadcast(b"hi" if c.rank() == 3 else b"", 3))
    assert res == [b"hi"] * 4
    res = run_threads(w, lambda c: c.all_gather(bytes([c.rank()])))
    assert res == [[bytes([0]), bytes([1]), bytes([2]), bytes([3])]] * 4

    def ring(c):
        n = c.world_size()
        c.send(bytes([c.rank()]), (c.rank() + 1) % n)
        return c.recv((c.rank() - 1) % n)

    assert run_threads(w, ring) == [bytes([3]), bytes([0]), bytes([1]), bytes([2])]


def test_local_world_fifo_and_timeout():
    w = local_world(2, 0.2)
    w[0].send(b"a", 1)
    w[0].send(b"b", 1)
    assert w[1].recv(0) == b"a" and w[1].recv(0) == b"b"
    with pytest.raises(CommTimeout):
        w[1].recv(0)


def test_local_world_topology_aware_exchange_real():
    topo = MeshTorusHybrid.new_2d(2, 4, 1)
    w = local_world(8, 10.0)
    comms = [TopologyAwareComm(c, topo) for c in w]
    res = run_threads(comms, lambda c: c.exchange_with_neighbors(bytes([c.rank()])))
    for r, got in enumerate(res):
        for peer, data in got:
            assert data == bytes([peer])
    res = run_threads(comms, lambda c: c.nearest_neighbor_exchange(bytes([c.rank()]), 1))
    for r, got in enumerate(res):
        x, y = r % 2, r // 2
        assert got == [bytes([((y + 1) % 4) * 2 + x]), bytes([((y - 1) % 4) * 2 + x])]
    res = run_threads(comms, lambda c: from_u64(c.reduce_on_group(u64(c.rank()), [0, 1, 2, 3], DType.U64))
                      if c.rank() < 4 else None)
    assert res[:4] == [6, 6, 6, 6]


def test_fault_plan_kill_rank_reaches_peers():
    plan = FaultPlan()
    plan.add(FaultRule(rank=1, at_op=1, op_kind="", action=FaultRule.Action.Kill))
    w = local_world(3, 5.0, plan)

    def body(c):
        c.all_reduce(u64(1), ReduceOp.Sum)   # op 0: everyone
        c.all_reduce(u64(1), ReduceOp.Sum)   # op 1: rank 1 dies here
        return "ok"

    res = run_threads(w, body)
    assert all(isinstance(r, CommError) for r in res), res


def test_fault_plan_drop_then_timeout():
    plan = FaultPlan()
    plan.add(FaultRule(rank=0, at_op=0, op_kind="send", action=FaultRule.Action.Drop))
    w = local_world(2, 0.3, plan)
    w[0].send(b"dropped", 1)
    w[0].send(b"second", 1)
    assert w[1].recv(0) == b"second"
    with pytest.raises(CommTimeout):
        w[1].recv(0)


def test_comm_scenario_on_local_world_threads():
    """The shared communicator workload (also run on the device backend on 2 GPUs)
    runs on host ranks and gives the reference's results."""
    import struct

    from comm_scenario import host_results
    from mtorus.core.topology import MeshTorusHybrid

    res = host_results(2, MeshTorusHybrid.new_2d(2, 1, 1))
    for r, o in enumerate(res):
        assert o["ar_u64_sum"] == struct.pack("<3Q", 3, 12, (2 ** 64 + 1) % 2 ** 64)
        assert o["ar_i32_mean"] == struct.pack("<3i", 4, -5, 100)
        assert o["ar_u8_sum"] == bytes([144, 1, 254, 6])
        assert o["bc"] == b"root says hi 1"
        assert o["ag"] == [b"x\x00", b"xx\x01"]
        assert o["p2p"] == [b"msg %d from %d" % (k, 1 - r) for k in range(3)]
        # the 2 x 1 torus: both x neighbours are the other rank, both y neighbours this rank itself
        assert o["exchange"] == [(1 - r, b"halo of %d" % (1 - r))] * 2 + [(r, b"halo of %d" % r)] * 2
        assert o["pc_rs"] == struct.pack("<2Q", 1 + 4 * r, 3 + 4 * r)
