"""One communicator workload, run unchanged on any backend: the reference's
collective and exchange cases (crates/mt-comm/src/collective.rs:39-53,
mock.rs:123-234, topology_aware.rs:155-292) as one sequence per rank.  The
results of the host LocalWorld run are the oracle for the device backend."""
import struct


def u64s(*v):
    return b"".join(struct.pack("<Q", x & (2 ** 64 - 1)) for x in v)


def scenario(comm, topo):
    from mtorus.comm import DType, ReduceOp, TopologyAwareComm
    from mtorus.core import CollectiveOp

    r, n = comm.rank(), comm.world_size()
    out = {}
    # all_reduce over every element type and op (reference: Sum over u64 by default)
    out["ar_u64_sum"] = comm.all_reduce(u64s(r + 1, 2 * r + 5, 2 ** 63 + r), ReduceOp.Sum, DType.U64)
    out["ar_u64_max"] = comm.all_reduce(u64s(r, 7 - r), ReduceOp.Max, DType.U64)
    out["ar_i64_min"] = comm.all_reduce(struct.pack("<3q", -r, r * 10, 5), ReduceOp.Min, DType.I64)
    out["ar_f32_sum"] = comm.all_reduce(struct.pack("<4f", 0.1 * (r + 1), 1e7, -3.25 * r, 1.0 / 3), ReduceOp.Sum,
                                        DType.F32)
    out["ar_f32_mean"] = comm.all_reduce(struct.pack("<2f", r + 0.5, -2.0 * r), ReduceOp.Mean, DType.F32)
    out["ar_f64_prod"] = comm.all_reduce(struct.pack("<2d", r + 1.5, -1.0), ReduceOp.Product, DType.F64)
    out["ar_i32_mean"] = comm.all_reduce(struct.pack("<3i", 7 * r + 1, -5, 100), ReduceOp.Mean, DType.I32)
    out["ar_u8_sum"] = comm.all_reduce(bytes([200, r, 255, 3]), ReduceOp.Sum, DType.U8)
    # rank 0's length sets the element count; a shorter message reads as zeros
    out["ar_ragged"] = comm.all_reduce(u64s(*range(4 - (r % 2))), ReduceOp.Sum, DType.U64)
    out["bc"] = comm.broadcast(b"root says hi %d" % r, n - 1)
    out["ag"] = comm.all_gather(b"x" * (r + 1) + bytes([r]))
    # point-to-point around the ring, three messages in flight per pair
    nxt, prv = (r + 1) % n, (r - 1) % n
    for k in range(3):
        comm.send(b"msg %d from %d" % (k, r), nxt)
    out["p2p"] = [comm.recv(prv) for _ in range(3)]
    comm.barrier()
    # the topology-aware wrapper over the same communicator
    t = TopologyAwareComm(comm, topo)
    out["exchange"] = t.exchange_with_neighbors(b"halo of %d" % r)
    out["nn_axis0"] = t.nearest_neighbor_exchange(b"axis0 from %d" % r, 0)
    out["pc_ar"] = t.perform_collective(CollectiveOp.AllReduce, u64s(r + 1, 10), DType.U64)
    out["pc_bc"] = t.perform_collective(CollectiveOp.Broadcast, b"b%d" % r, DType.U64)
    out["pc_ag"] = t.perform_collective(CollectiveOp.AllGather, b"g%d" % r, DType.U64)
    out["pc_rs"] = t.perform_collective(CollectiveOp.ReduceScatter, u64s(*[r + k for k in range(2 * n)]),
                                        DType.U64)
    return out


def host_results(n, topo):
    """The oracle: the scenario on n LocalWorld ranks (one thread each)."""
    from mtorus.comm import local_world, run_threads

    comms = local_world(n, 30.0)
    res = run_threads(comms, scenario, topo)
    for x in res:
        if isinstance(x, BaseException):
            raise x
    return res
