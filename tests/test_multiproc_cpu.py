"""Multi-process (gloo, world 2-4) tests of the torch.distributed communicator, the
multi-rank pipeline executor and the data-parallel bucket reducer."""
import pytest
import torch

from dist_util import run_dist


def _comm_body(rank, world):
    from mtorus.comm import DType, ReduceOp, TopologyAwareComm, from_u64, u64
    from mtorus.comm.nccl import DistCommunicator
    from mtorus.core.coordinator import CollectiveOp
    from mtorus.core.topology import MeshTorusHybrid

    c = DistCommunicator()
    out = {"sum": from_u64(c.all_reduce(u64(rank + 1), ReduceOp.Sum)),
           "max": from_u64(c.all_reduce(u64(rank + 1), ReduceOp.Max)),
           "bcast": c.broadcast(b"root" if rank == 1 else b"", 1),
           "gather": c.all_gather(bytes([rank] * (rank + 1)))}
    peer = (rank + 1) % world
    c.send(bytes([rank, 7]), peer)
    out["recv"] = c.recv((rank - 1) % world)
    t = TopologyAwareComm(c, MeshTorusHybrid.new_2d(world, 1, 1))
    out["halo"] = t.nearest_neighbor_exchange(bytes([rank]), 0)
    out["rs"] = t.perform_collective(CollectiveOp.ReduceScatter, u64(1) * world)
    return out


def test_dist_communicator_gloo():
    res = run_dist(_comm_body, 3)
    for r, o in enumerate(res):
        assert o["sum"] == 6 and o["max"] == 3 and o["bcast"] == b"root"
        assert o["gather"] == [bytes([k] * (k + 1)) for k in range(3)]
        assert o["recv"] == bytes([(r - 1) % 3, 7])
        assert o["halo"] == [bytes([(r + 1) % 3]), bytes([(r - 1) % 3])]
        assert o["rs"] == (3).to_bytes(8, "little")


def _make_stages(seed=0):
    torch.manual_seed(seed)
    return [torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.Tanh()),
            torch.nn.Sequential(torch.nn.Linear(16, 16), torch.nn.Tanh()),
            torch.nn.Sequential(torch.nn.Linear(16, 4))]


def _pp_body(rank, world, sched_name, ckpt_name):
    from mtorus.pipeline import CheckpointStrategy, DistributedPipelineExecutor, ScheduleType

    stages = _make_stages()
    M = 4
    g = torch.Generator().manual_seed(1)
    xs = [torch.randn(2, 8, generator=g) for _ in range(M)]
    ys = [torch.randn(2, 4, generator=g) for _ in range(M)]
    shapes = [(2, 16), (2, 16), (2, 4)]
    ex = DistributedPipelineExecutor(stages[rank], list(range(world)), getattr(ScheduleType, sched_name), M,
                                     getattr(CheckpointStrategy, ckpt_name),
                                     loss_fn=torch.nn.functional.mse_loss, act_shape=shapes[max(rank - 1, 0)])
    losses = ex.run(xs if rank == 0 else None, ys if rank == world - 1 else None)
    grads = [p.grad.clone() for p in stages[rank].parameters()]
    return losses, grads


@pytest.mark.parametrize("sched", ["OneF1B", "Gpipe"])
@pytest.mark.parametrize("ckpt", ["None_", "Full"])
def test_pipeline_executor_matches_single_process(sched, ckpt):
    res = run_dist(_pp_body, 3, (sched, ckpt))
    stages = _make_stages()
    M = 4
    g = torch.Generator().manual_seed(1)
    xs = [torch.randn(2, 8, generator=g) for _ in range(M)]
    ys = [torch.randn(2, 4, generator=g) for _ in range(M)]
    ref_losses = []
    for x, y in zip(xs, ys):
        out = stages[2](stages[1](stages[0](x)))
        loss = torch.nn.functional.mse_loss(out, y) / M
        loss.backward()
        ref_losses.append(loss.item() * M)
    assert all(abs(a - b) < 1e-5 for a, b in zip(res[2][0], ref_losses))
    for r in range(3):
        for gp, p in zip(res[r][1], stages[r].parameters()):
            assert torch.allclose(gp, p.grad, atol=1e-5), (r, (gp - p.grad).abs().max())


def _dp_body(rank, world):
    from mtorus.parallel.data_parallel import NcclBucketReducer
    from mtorus.parallel.flat import FlatParams

    torch.manual_seed(0)
    m = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.Linear(32, 8))
    flat = FlatParams([[p] for p in m.parameters()], "cpu", with_w16=False)
    red = NcclBucketReducer(flat, None, bucket_bytes=1024)
    for p in m.parameters():
        p.main_grad.fill_(float(rank + 1))
    for p in reversed(list(m.parameters())):
        red.on_ready([p])
    red.finish()
    return flat.grad.clone(), len(red.plan)


def test_bucket_reducer_averages_across_ranks():
    res = run_dist(_dp_body, 2)
    for g, nb in res:
        assert nb > 1 and torch.allclose(g[g != 0], torch.full_like(g[g != 0], 1.5))
