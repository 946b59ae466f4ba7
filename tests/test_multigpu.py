"""Multi-GPU tests (NCCL process group, one process per GPU; skipped with < 2 GPUs):
the fused NVLink collectives and the fused data-parallel training step against
the NCCL baseline."""
import pytest
import torch

from dist_util import run_dist

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _ngpu():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


needs2 = pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")


def _coll_body(rank, world):
    import torch

    from mtorus.core.topology import MeshTorusHybrid
    from mtorus.parallel.symm import SymmCollectives, halo_plan

    torch.cuda.set_device(rank)
    c = SymmCollectives(f"cuda:{rank}", max_bytes=1 << 22)
    out = {}
    n = 1000 * 8
    c.buf.tensor[:n] = torch.arange(n, device="cuda", dtype=torch.float32) * (rank + 1)
    out["ar"] = c.all_reduce(n).clone().cpu()
    c.buf.tensor.view(torch.bfloat16)[:n] = (torch.ones(n, device="cuda") * (rank + 1)).bfloat16()
    out["ar16"] = c.all_reduce(n, torch.bfloat16).float().clone().cpu()
    c.buf.tensor[:256] = rank + 1.0
    c.all_gather(256 * 4)
    out["ag"] = c.recv.tensor[:256 * world].clone().cpu()
    c.buf.tensor[:256] = 7.0 if rank == 1 else -1.0
    c.broadcast(256 * 4, root=1)
    out["bc"] = c.buf.tensor[:256].clone().cpu()
    topo = MeshTorusHybrid.new_2d(world, 1, 1)
    nr, ns = halo_plan(topo, rank, "cuda")
    c.buf.tensor[:64] = float(rank)
    c.halo(64 * 4, nr, ns)
    out["halo"] = c.recv.tensor[:64 * 4].clone().cpu()
    out["status"] = c.ctx.status()
    torch.cuda.synchronize()
    return out


@needs2
def test_symm_collectives_2gpu():
    res = run_dist(_coll_body, 2, backend="nccl")
    n = 8000
    base = torch.arange(n, dtype=torch.float32)
    for r, o in enumerate(res):
        assert o["status"] == 0
        assert torch.allclose(o["ar"], base * 3)
        assert torch.allclose(o["ar16"], torch.full((n,), 3.0))
        assert torch.equal(o["ag"], torch.cat([torch.full((256,), 1.0), torch.full((256,), 2.0)]))
        assert torch.equal(o["bc"], torch.full((256,), 7.0))
        # 2-wide torus: the single peer's + and - messages land in two distinct slots
        peer = 1 - r
        assert torch.equal(o["halo"][:128], torch.full((128,), float(peer)))


def _dp_body(rank, world, dp):
    import torch

    from mtorus.models.gpt import GptConfig
    from mtorus.training.engine import GptTrainer

    torch.cuda.set_device(rank)
    cfg = GptConfig(vocab_size=512, d_model=256, num_layers=2, num_heads=2, d_ff=1024, max_seq_len=128,
                    dropout=0.0)
    tr = GptTrainer(cfg, device=f"cuda:{rank}", lr=1e-3, init="normal", seed=0, dp=dp, bucket_mb=0.5)
    g = torch.Generator().manual_seed(100 + rank)
    losses = []
    for _ in range(4):
        t = torch.randint(0, cfg.vocab_size, (2, 129), generator=g)
        losses.append(tr.train_step(t[:, :-1].contiguous().pin_memory(), t[:, 1:].contiguous().pin_memory()))
    w = tr.flat.w16[:4096].float().cpu()
    st = 0
    if dp == "symm":
        st = tr.reducer.ctx.status()
    return losses, w, st


@needs2
def test_fused_dp_matches_nccl_baseline():
    a = run_dist(_dp_body, 2, ("nccl",), backend="nccl")
    b = run_dist(_dp_body, 2, ("symm",), backend="nccl")
    for r in range(2):
        assert b[r][2] == 0
        for x, y in zip(a[r][0], b[r][0]):
            assert abs(x - y) < 2e-2 * max(1.0, abs(x)), (a[r][0], b[r][0])
        assert torch.allclose(a[r][1], b[r][1], atol=2e-2, rtol=2e-2)
    # every rank holds the same weights after the all-gather
    assert torch.equal(b[0][1], b[1][1])
