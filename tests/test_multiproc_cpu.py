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


def _pp_body(rank, world, sched_name, ckpt_name, wire="native"):
    from mtorus.pipeline import CheckpointStrategy, DistributedPipelineExecutor, ScheduleType

    stages = _make_stages()
    M = 4
    g = torch.Generator().manual_seed(1)
    xs = [torch.randn(2, 8, generator=g) for _ in range(M)]
    ys = [torch.randn(2, 4, generator=g) for _ in range(M)]
    shapes = [(2, 16), (2, 16), (2, 4)]
    ex = DistributedPipelineExecutor(stages[rank], list(range(world)), getattr(ScheduleType, sched_name), M,
                                     getattr(CheckpointStrategy, ckpt_name),
                                     loss_fn=torch.nn.functional.mse_loss, act_shape=shapes[max(rank - 1, 0)],
                                     wire=wire)
    losses = ex.run(xs if rank == 0 else None, ys if rank == world - 1 else None)
    grads = [p.grad.clone() for p in stages[rank].parameters()]
    return losses, grads


@pytest.mark.parametrize("sched", ["OneF1B", "Gpipe"])
@pytest.mark.parametrize("ckpt", ["None_", "Full", "Selective"])
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


def test_pipeline_executor_fp8_wire_tracks_full_precision():
    """Stage transfers as block-scaled FP8 (E4M3 activations, E5M2 gradients; the
    reference compresses them in PipelineComm, communicator.rs:44-73): losses and
    gradients stay within FP8 rounding of the full-precision run."""
    ref = run_dist(_pp_body, 3, ("OneF1B", "None_"))
    got = run_dist(_pp_body, 3, ("OneF1B", "None_", "fp8"))
    for a, b in zip(got[2][0], ref[2][0]):
        assert abs(a - b) <= 0.05 * abs(b) + 1e-4
    for r in range(3):
        for ga, gb in zip(got[r][1], ref[r][1]):
            assert float((ga - gb).norm()) <= 0.15 * float(gb.norm()) + 1e-6, r


class _Counting(torch.nn.Module):
    def __init__(self, d):
        super().__init__()
        self.lin = torch.nn.Linear(d, d)
        self.calls = 0

    def forward(self, x):
        self.calls += 1
        return torch.tanh(self.lin(x))


def _selective_body(rank, world, ckpt_name):
    from mtorus.pipeline import CheckpointStrategy, DistributedPipelineExecutor, ScheduleType

    torch.manual_seed(3)
    stage = torch.nn.Sequential(*[_Counting(8) for _ in range(4)])
    M = 3
    g = torch.Generator().manual_seed(4)
    xs = [torch.randn(2, 8, generator=g) for _ in range(M)]
    ys = [torch.randn(2, 8, generator=g) for _ in range(M)]
    ex = DistributedPipelineExecutor(stage, [0], ScheduleType.OneF1B, M, getattr(CheckpointStrategy, ckpt_name),
                                     loss_fn=torch.nn.functional.mse_loss, act_shape=(2, 8))
    ex.run(xs, ys)
    return [m.calls for m in stage], [p.grad.clone() for p in stage.parameters()]


def test_selective_checkpointing_recomputes_only_the_second_half():
    """Selective (reference checkpoint.rs:43-60 splits the stage's layers at len / 2):
    the first half runs once per micro-batch, the second half once more in backward,
    and the gradients are those of the plain stage."""
    calls_sel, grads_sel = run_dist(_selective_body, 1, ("Selective",))[0]
    calls_none, grads_none = run_dist(_selective_body, 1, ("None_",))[0]
    calls_full, _ = run_dist(_selective_body, 1, ("Full",))[0]
    assert calls_none == [3, 3, 3, 3]
    assert calls_sel == [3, 3, 6, 6]
    assert calls_full == [6, 6, 6, 6]
    for a, b in zip(grads_sel, grads_none):
        assert torch.allclose(a, b, atol=1e-6)


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


def _gpt_dppp_body(rank, world):
    """2 replicas x 2 pipeline stages of the reference-path GPT on gloo: the layout of
    PipelineLayout, activations and gradients on separate groups, DP averaging."""
    import torch.distributed as dist

    from mtorus.models.gpt import GptConfig, GptModel
    from mtorus.pipeline import CheckpointStrategy, DistributedPipelineExecutor, ScheduleType
    from mtorus.training.pipeline_engine import PipelineLayout

    cfg = GptConfig(vocab_size=64, d_model=32, num_layers=2, num_heads=2, d_ff=64, max_seq_len=16, dropout=0.0)
    lay = PipelineLayout(2, 2)
    replica, stage = lay.coords(rank)
    groups = {}
    for ranks in lay.stage_ranks:
        ga, gg = dist.new_group(ranks), dist.new_group(ranks)
        if rank in ranks:
            groups["act"], groups["grad"] = ga, gg
    for ranks in lay.dp_ranks:
        g = dist.new_group(ranks)
        if rank in ranks:
            groups["dp"] = g
    torch.manual_seed(0)
    full = GptModel(cfg)
    sd = full.state_dict()
    m = GptModel(cfg, layers=(stage, stage + 1), embed=stage == 0, head=stage == 1)
    own = m.state_dict()
    for k in own:
        g = f"blocks.{int(k.split('.')[1]) + stage}.{k.split('.', 2)[2]}" if k.startswith("blocks.") else k
        own[k].copy_(sd[g])
    M, b, S = 4, 2, 16
    gen = torch.Generator().manual_seed(10 + replica)
    t = torch.randint(0, cfg.vocab_size, (M, b, S + 1), generator=gen)
    ids, tgt = list(t[..., :-1].unbind(0)), list(t[..., 1:].unbind(0))

    def loss_fn(logits, y):
        return torch.nn.functional.cross_entropy(logits.reshape(-1, cfg.vocab_size), y.reshape(-1))

    ex = DistributedPipelineExecutor(m, lay.stage_ranks[replica], ScheduleType.OneF1B, M, CheckpointStrategy.Full,
                                     loss_fn=loss_fn, act_shape=(b, S, cfg.d_model), stage_fn=m.forward_stage,
                                     group=groups["act"], grad_group=groups["grad"])
    losses = ex.run(ids if stage == 0 else None, tgt if stage == 1 else None)
    for p in m.parameters():
        dist.all_reduce(p.grad, group=groups["dp"])
        p.grad /= 2
    names = {}
    for k, p in m.named_parameters():
        g = f"blocks.{int(k.split('.')[1]) + stage}.{k.split('.', 2)[2]}" if k.startswith("blocks.") else k
        names[g] = p.grad.clone()
    return {"losses": losses, "grads": names}


def test_gpt_dp2_pp2_gloo_matches_single_process():
    from mtorus.models.gpt import GptConfig, GptModel

    res = run_dist(_gpt_dppp_body, 4)
    cfg = GptConfig(vocab_size=64, d_model=32, num_layers=2, num_heads=2, d_ff=64, max_seq_len=16, dropout=0.0)
    torch.manual_seed(0)
    full = GptModel(cfg)
    M, b, S = 4, 2, 16
    total = 0.0
    for replica in range(2):
        gen = torch.Generator().manual_seed(10 + replica)
        t = torch.randint(0, cfg.vocab_size, (M, b, S + 1), generator=gen)
        logits = full(t[..., :-1].reshape(M * b, S))
        loss = torch.nn.functional.cross_entropy(logits.reshape(-1, cfg.vocab_size), t[..., 1:].reshape(-1))
        (loss / 2).backward()
        total += float(loss)
    got = {}
    for r in res:
        got.update(r["grads"])
    assert set(got) == {n for n, _ in full.named_parameters()}
    for n, p in full.named_parameters():
        assert torch.allclose(got[n], p.grad, rtol=1e-4, atol=1e-6), n
    # last stages (ranks 1 and 3) report each replica's micro-batch losses
    mean_loss = (sum(res[1]["losses"]) + sum(res[3]["losses"])) / 8
    assert abs(mean_loss - total / 2) < 1e-4


def _dp_e5m2_body(rank, world):
    from mtorus.parallel.data_parallel import NcclBucketReducer
    from mtorus.parallel.flat import FlatParams

    torch.manual_seed(0)
    m = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.Linear(32, 40), torch.nn.Linear(40, 8))
    flat = FlatParams([[p] for p in m.parameters()], "cpu", with_w16=False)
    red = NcclBucketReducer(flat, None, bucket_bytes=1024, grad_fp8=True)
    g = torch.Generator().manual_seed(10 + rank)
    for p in m.parameters():
        p.main_grad.copy_(torch.randn(p.main_grad.shape, generator=g) * 10.0 ** (rank - 2))
    before = flat.grad.clone()
    for p in reversed(list(m.parameters())):
        red.on_ready([p])
    red.finish()
    return before, flat.grad.clone(), [tuple(r) for r in red.plan.ranges]


@pytest.mark.parametrize("world", [2, 3])
def test_bucket_reducer_e5m2_transport(world):
    """E5M2 transport through the NCCL-style reducer (gloo here): every rank ends with
    the same bytes, equal to the bf16-rounded mean of the E5M2-decoded gradients."""
    from mtorus.parallel.data_parallel import e5m2_decode, e5m2_encode

    res = run_dist(_dp_e5m2_body, world)
    inputs = [r[0] for r in res]
    for r in res[1:]:
        assert torch.equal(r[1], res[0][1])  # identical on every rank
    out = res[0][1]
    for s, e in res[0][2]:
        L = e - s
        pad = (-L) % 32
        dec = [e5m2_decode(*e5m2_encode(torch.cat([x[s:e], torch.zeros(pad)])))[:L] for x in inputs]
        ref = (sum(dec) * (1.0 / world)).to(torch.bfloat16).float()
        assert torch.equal(out[s:e], ref)
        exact = sum(x[s:e] for x in inputs) / world
        assert float((out[s:e] - exact).norm() / exact.norm()) < 0.1
