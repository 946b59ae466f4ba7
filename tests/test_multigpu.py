"""Multi-GPU tests (NCCL process group, one process per GPU; skipped with < 2 GPUs):
the fused NVLink collectives and the fused data-parallel training step against
the NCCL baseline."""
import os

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


def _dp_body(rank, world, dp, nvls=False, ag_mc=False):
    import os

    import torch

    if nvls:
        os.environ["MTORUS_DP_NVLS"] = "1"
    if ag_mc:
        os.environ["MTORUS_DP_AG_MC"] = "1"
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
        if (nvls and not tr.reducer.nvls) or (ag_mc and not tr.opt.w16_mc):
            st = -1  # no multicast binding on this fabric: nothing to compare
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


@needs2
def test_fused_dp_nvls_reduce_scatter_matches_peer_loads():
    """The NVLS (multimem.ld_reduce) bucket reduce-scatter gives the same training
    trajectory as the peer-load one."""
    a = run_dist(_dp_body, 2, ("symm",), backend="nccl")
    b = run_dist(_dp_body, 2, ("symm", True), backend="nccl")
    if b[0][2] == -1:
        pytest.skip("no NVLink multicast on this fabric")
    for r in range(2):
        assert b[r][2] == 0
        for x, y in zip(a[r][0], b[r][0]):
            assert abs(x - y) < 2e-2 * max(1.0, abs(x)), (a[r][0], b[r][0])
        assert torch.allclose(a[r][1], b[r][1], atol=2e-2, rtol=2e-2)


def _dp_graph_body(rank, world, dp, fp8):
    import gc

    import torch

    from mtorus.models.gpt import GptConfig
    from mtorus.training.engine import GptTrainer

    torch.cuda.set_device(rank)
    dev = f"cuda:{rank}"
    cfg = GptConfig(vocab_size=512, d_model=256, num_layers=2, num_heads=2, d_ff=1024, max_seq_len=128,
                    dropout=0.0)
    g = torch.Generator().manual_seed(300 + rank)
    data = [torch.randint(0, cfg.vocab_size, (2, 129), generator=g) for _ in range(6)]
    ids = [t[:, :-1].contiguous().to(dev) for t in data]
    tgt = [t[:, 1:].contiguous().to(dev) for t in data]
    out = {}
    for graph in (False, True):
        tr = GptTrainer(cfg, device=dev, lr=1e-3, init="normal", seed=0, dp=dp, bucket_mb=0.5, fp8=fp8)
        losses = []
        for i in range(6):
            if graph and i == 2:
                tr.capture(ids[i], tgt[i])
            loss = tr.graph_step(ids[i], tgt[i]) if graph and i >= 2 else tr.step_device(ids[i], tgt[i])
            losses.append(float(loss))
        torch.cuda.synchronize()
        st = tr.reducer.ctx.status() if dp == "symm" else 0
        out[graph] = (losses, tr.flat.w16[:4096].float().cpu(), st)
        del tr  # a graph holding NCCL calls is released before the group is destroyed
        gc.collect()
    return out


@needs2
@pytest.mark.parametrize("dp,fp8", [("symm", False), ("symm", True), ("nccl", True)])
def test_captured_dp_step_replays_like_eager(dp, fp8):
    """The whole data-parallel step captured once as a CUDA graph and replayed: the
    fused path's flag epochs and amax stamps come from device step counters, so
    four replays follow the eager trajectory."""
    res = run_dist(_dp_graph_body, 2, (dp, fp8), backend="nccl")
    for o in res:
        (le, we, se), (lg, wg, sg) = o[False], o[True]
        assert se == 0 and sg == 0
        for x, y in zip(le, lg):
            assert abs(x - y) < 1e-2 * max(1.0, abs(x)), (le, lg)
        assert torch.allclose(we, wg, atol=1e-2, rtol=1e-2)
    assert torch.equal(res[0][True][1], res[1][True][1])


def _pp_body(rank, world, sched_name, ckpt_name):
    import torch

    from mtorus.models.gpt import GptConfig, GptModel
    from mtorus.pipeline import CheckpointStrategy, ScheduleType
    from mtorus.training.pipeline_engine import PipelineTrainer

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    cfg = GptConfig(vocab_size=512, d_model=256, num_layers=4, num_heads=2, d_ff=1024, max_seq_len=128,
                    dropout=0.0)
    M, b, S = 4, 2, 128
    torch.manual_seed(0)
    full = GptModel(cfg)
    full.init_normal_(0.02)
    sd = {k: v.clone() for k, v in full.state_dict().items()}
    tr = PipelineTrainer(cfg, pp=world, dp=1, schedule=getattr(ScheduleType, sched_name), num_microbatches=M,
                         micro_batch=b, seq_len=S, checkpoint=getattr(CheckpointStrategy, ckpt_name), fp8=False,
                         lr=1e-3, device=dev)
    tr.load_global_state_dict(sd)
    g = torch.Generator().manual_seed(7)
    t = torch.randint(0, cfg.vocab_size, (M, b, S + 1), generator=g)
    ids, tgt = t[:, :, :-1].contiguous(), t[:, :, 1:].contiguous()
    loss = tr.forward_backward(list(ids.to(dev).unbind(0)), list(tgt.to(dev).unbind(0)))
    grads = {tr.global_name(n): p.main_grad.float().cpu().clone() for n, p in tr.model.named_parameters()}
    out = {"loss": None if loss is None else float(loss), "grads": grads}
    if rank == 0:
        # single-GPU fused model on the whole batch: mean loss over all micro-batch tokens
        ref = GptModel(cfg).to(dev)
        ref.load_state_dict(sd)
        ref.flatten(dev)
        l_ref = ref.fused_loss(ids.reshape(M * b, S).to(dev), tgt.reshape(M * b, S).to(dev))
        l_ref.backward()
        out["ref_loss"] = float(l_ref)
        out["ref_grads"] = {n: p.main_grad.float().cpu().clone() for n, p in ref.named_parameters()}
    # a full optimizer step runs and the pipeline-wide overflow flag stays clear
    tr.optimizer_step()
    out["skip"] = float(tr.opt.state[5])
    torch.cuda.synchronize()
    return out


@needs2
@pytest.mark.parametrize("sched,ckpt", [("OneF1B", "Full"), ("Gpipe", "None_")])
def test_pipeline_trainer_matches_single_gpu(sched, ckpt):
    res = run_dist(_pp_body, 2, (sched, ckpt), backend="nccl")
    ref_loss, ref_grads = res[0]["ref_loss"], res[0]["ref_grads"]
    assert abs(res[1]["loss"] - ref_loss) < 2e-2 * abs(ref_loss)
    checked = 0
    for r in range(2):
        assert res[r]["skip"] == 0.0
        for name, gr in res[r]["grads"].items():
            gref = ref_grads[name]
            err = (gr - gref).norm() / max(gref.norm(), 1e-6)
            assert err < 5e-2, (r, name, float(err))
            checked += 1
    assert checked == len(ref_grads)


@needs2
def test_fused_dp_multicast_weight_allgather_matches_peer_stores():
    """The sharded Adam storing the new weights once through the multicast address (the
    default from 4 ranks up) gives the same trajectory and bit-identical weights on every
    rank as storing them into each peer."""
    a = run_dist(_dp_body, 2, ("symm",), backend="nccl")
    b = run_dist(_dp_body, 2, ("symm", False, True), backend="nccl")
    if b[0][2] == -1:
        pytest.skip("no NVLink multicast on this fabric")
    for r in range(2):
        assert b[r][2] == 0
        for x, y in zip(a[r][0], b[r][0]):
            assert abs(x - y) < 2e-2 * max(1.0, abs(x)), (a[r][0], b[r][0])
        assert torch.allclose(a[r][1], b[r][1], atol=2e-2, rtol=2e-2)
    assert torch.equal(b[0][1], b[1][1])


def _amax_body(rank, world, kind):
    import torch

    from mtorus.ops import fp8 as F8

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    st = F8.Fp8State(dev, history=4, capacity=64)
    st.set_amax_sync(F8.SymmAmaxSync(dev, st.cap) if kind == "symm" else F8.NcclAmaxSync())
    out = {"scale": [], "codes_match": []}
    for step in range(3):
        torch.manual_seed(100 * step + rank)
        xs = {"a": (torch.randn(4096, 256) * (rank + 1) * (step + 1)).to(dev),
              "b": (torch.randn(1000, 8) * (2.0 - rank)).to(dev)}
        for name, x in xs.items():
            x = x.bfloat16()
            q, _ = st.quantize(x, name, F8.E4M3 if name == "a" else F8.E5M2)
            s = st.names[name]
            ref = F8.quantize(x, st.fmts[s], st.scale[s:s + 1])
            out["codes_match"].append(bool(torch.equal(q, ref)))
        st.end_step()
        out["scale"].append(st.scale[:2].cpu().clone())
    torch.cuda.synchronize()
    return out


@needs2
@pytest.mark.parametrize("kind", ["symm", "nccl"])
def test_fp8_amax_allreduce_2gpu(kind):
    """Delayed-scaling amax reduced over ranks: both ranks end every step with the
    same scales, equal to fmax / (max over ranks and history of amax); the fused
    quantise kernel writes the same codes as the plain one."""
    res = run_dist(_amax_body, 2, (kind,), backend="nccl")
    for o in res:
        assert all(o["codes_match"])
    for step in range(3):
        assert torch.equal(res[0]["scale"][step], res[1]["scale"][step])
    # step 3 (index 2): role "a" amax = max over ranks = 2 * 3 * max|randn|; scale = 416 / that (history 4)
    a_amax = [0.0, 0.0]
    for step in range(3):
        for r in range(2):
            torch.manual_seed(100 * step + r)
            xa = (torch.randn(4096, 256) * (r + 1) * (step + 1)).bfloat16().float()
            a_amax[0] = max(a_amax[0], float(xa.abs().max()))
    assert abs(float(res[0]["scale"][2][0]) - 416.0 / a_amax[0]) < 1e-3 * 416.0 / a_amax[0]


def _nvls_body(rank, world):
    import torch

    from mtorus.parallel.symm import SymmCollectives

    torch.cuda.set_device(rank)
    c = SymmCollectives(f"cuda:{rank}", max_bytes=1 << 22)
    out = {"nvls": c.nvls}
    n = 4096
    # FP8 all-reduce (peer loads): codes of small integers sum exactly
    vals = torch.full((n,), float(rank + 1), device="cuda").to(torch.float8_e4m3fn)
    c.buf.tensor.view(torch.uint8)[:n] = vals.view(torch.uint8)
    r8 = c.all_reduce_fp8(n, 0).clone().view(torch.float8_e4m3fn).float().cpu()
    out["fp8"] = r8
    if c.nvls:
        c.buf.tensor[:n] = torch.arange(n, device="cuda", dtype=torch.float32) * (rank + 1)
        out["ar"] = c.all_reduce_nvls(n).clone().cpu()
        c.buf.tensor.view(torch.bfloat16)[:n] = (torch.ones(n, device="cuda") * (rank + 1)).bfloat16()
        out["ar16"] = c.all_reduce_nvls(n, torch.bfloat16).float().clone().cpu()
        c.buf.tensor[:256] = 5.0 if rank == 1 else -1.0
        c.broadcast_nvls(256 * 4, root=1)
        out["bc"] = c.buf.tensor[:256].clone().cpu()
    out["status"] = c.ctx.status()
    torch.cuda.synchronize()
    return out


@needs2
def test_nvls_and_fp8_collectives_2gpu():
    res = run_dist(_nvls_body, 2, backend="nccl")
    n = 4096
    for o in res:
        assert o["status"] == 0
        assert torch.equal(o["fp8"], torch.full((n,), 3.0))
        if o["nvls"]:
            assert torch.allclose(o["ar"], torch.arange(n, dtype=torch.float32) * 3)
            assert torch.allclose(o["ar16"], torch.full((n,), 3.0))
            assert torch.equal(o["bc"], torch.full((256,), 5.0))


def _gather_gemm_body(rank, world):
    import torch

    from mtorus.ops import fp8 as F8
    from mtorus.parallel.symm import GatheredOperand

    torch.cuda.set_device(rank)
    dev = f"cuda:{rank}"
    M, N, K = 512, 768, 512
    g = torch.Generator().manual_seed(11)  # the same full operands on every rank
    b_full = (torch.randn(N, K, generator=g) * 0.5).to(torch.float8_e4m3fn).view(torch.uint8).to(dev)
    bt_full = b_full.t().contiguous()  # [K, N] for the MN-major (dgrad-style) use
    a = (torch.randn(M, K, generator=g)).to(torch.float8_e4m3fn).view(torch.uint8).to(dev)
    one = torch.ones(1, device=dev)
    out = {}
    w = GatheredOperand(N, K, dev)
    w.local_shard().copy_(b_full[w.lo:w.hi])  # each rank writes only its own rows
    w.publish()
    ref = F8.gemm_fp8(a, 0, b_full, 0, alpha=one)
    out["kmajor"] = torch.equal(w.gemm(a, 0, 0, alpha=one, method="direct"), ref)
    out["kmajor_overlap"] = torch.equal(w.gemm(a, 0, 0, alpha=one, method="overlap"), ref)
    wt = GatheredOperand(K, N, dev)  # B stored [K, N], sharded along K
    wt.local_shard().copy_(bt_full[wt.lo:wt.hi])
    wt.publish()
    out["mnmajor"] = torch.equal(wt.gemm(a, 0, 0, b_mn=True, alpha=one, method="direct"),
                                 F8.gemm_fp8(a, 0, bt_full, 0, b_mn=True, alpha=one))
    ref32 = F8.gemm_fp8(a, 0, bt_full, 0, b_mn=True, alpha=one, out_dtype=torch.float32)
    got32 = wt.gemm(a, 0, 0, b_mn=True, alpha=one, method="overlap", out_dtype=torch.float32)
    out["mnmajor_overlap_err"] = float((got32 - ref32).abs().max() / ref32.abs().max())
    w.retire()
    wt.retire()
    out["status"] = w.ctx.status()
    torch.cuda.synchronize()
    return out


@needs2
def test_gather_b_gemm_matches_local_gemm_2gpu():
    """Weight all-gather fused into the GEMM: a GEMM that reads each B tile from the rank owning it equals
    the same GEMM on a locally gathered B, bit for bit (same kernel, same tiles)."""
    for o in run_dist(_gather_gemm_body, 2, backend="nccl"):
        assert o["status"] == 0
        assert o["kmajor"] and o["mnmajor"] and o["kmajor_overlap"]
        assert o["mnmajor_overlap_err"] < 1e-5  # per-shard partial sums: fp32 summation order differs


def _bc_scatter_body(rank, world):
    import torch

    from mtorus.parallel.symm import SymmCollectives

    torch.cuda.set_device(rank)
    c = SymmCollectives(f"cuda:{rank}", max_bytes=1 << 22)
    out = {"nvls": c.nvls}
    if c.nvls:
        n = 1040 // 4  # two uneven chunks (528 + 512 bytes)
        c.buf.tensor[:n] = (torch.arange(n, device="cuda", dtype=torch.float32) + 7) if rank == 1 else -1.0
        c.broadcast_scatter_nvls(n * 4, root=1)
        out["bc"] = c.buf.tensor[:n].clone().cpu()
    out["status"] = c.ctx.status()
    torch.cuda.synchronize()
    return out


@needs2
def test_broadcast_scatter_multicast_2gpu():
    for o in run_dist(_bc_scatter_body, 2, backend="nccl"):
        assert o["status"] == 0
        if o["nvls"]:
            assert torch.equal(o["bc"], torch.arange(260, dtype=torch.float32) + 7)


def _e5m2_rs_body(rank, world):
    import torch

    from mtorus._ext import cuda as _cuda
    from mtorus.parallel.symm import SymmBuffer, SymmContext, _chunk_len

    torch.cuda.set_device(rank)
    dev = f"cuda:{rank}"
    n = 8192
    ctx = SymmContext(dev, num_slots=16)
    grad = SymmBuffer(n, torch.float32, dev)
    codes = SymmBuffer(n, torch.uint8, dev)
    sf = SymmBuffer(n // 32, torch.uint8, dev)
    g = torch.Generator().manual_seed(50 + rank)
    mine = torch.randn(n, generator=g) * torch.logspace(-6, 2, n // 32).repeat_interleave(32)
    grad.tensor.copy_(mine)
    st = torch.zeros(16, device=dev)
    clen = _chunk_len(n, world)
    _cuda().dp_quant_e5m2(grad.tensor.data_ptr(), codes.tensor.data_ptr(), sf.tensor.data_ptr(), n)
    _cuda().symm_rs_bucket_e5m2(codes.ptrs, sf.ptrs, ctx.flags.ptrs, rank, 0, n, clen, 3, 1, st, 16, 1.0 / world,
                                grad.tensor.data_ptr())
    torch.cuda.synchronize()
    lo, hi = rank * clen, min(n, (rank + 1) * clen)
    return {"input": mine, "chunk": grad.tensor[lo:hi].cpu(), "lo": lo, "hi": hi, "sumsq": float(st[0]),
            "bad": float(st[1]), "status": ctx.status()}


@needs2
def test_e5m2_gradient_reduce_scatter_2gpu():
    """Each rank's chunk is the mean over ranks of the E5M2-encoded gradients (the
    MX block rule with 32-value blocks), decoded exactly as the PyTorch oracle does."""
    from mtorus.ops.mxfp8 import E5M2, mx_dequantize, mx_quantize_ref

    res = run_dist(_e5m2_rs_body, 2, backend="nccl")
    decoded = [mx_dequantize(mx_quantize_ref(o["input"].reshape(-1, 32), E5M2)).reshape(-1) for o in res]
    mean = sum(decoded) / len(decoded)
    for o in res:
        assert o["status"] == 0 and o["bad"] == 0.0
        ref = mean[o["lo"]:o["hi"]]
        assert torch.allclose(o["chunk"], ref, rtol=1e-6, atol=0.0)
        assert abs(o["sumsq"] - float((ref.double() ** 2).sum())) <= 1e-4 * float((ref.double() ** 2).sum())
        # and within E5M2 precision of the exact fp32 mean
        exact = sum(r["input"] for r in res)[o["lo"]:o["hi"]] / len(res)
        assert float((o["chunk"] - exact).norm() / exact.norm()) < 0.1



def _device_comm_body(rank, world):
    import torch

    from comm_scenario import scenario
    from mtorus.comm.device import SymmCommunicator
    from mtorus.core.topology import MeshTorusHybrid

    torch.cuda.set_device(rank)
    comm = SymmCommunicator(device=f"cuda:{rank}", max_bytes=1 << 16, tensor_bytes=1 << 20)
    out = scenario(comm, MeshTorusHybrid.new_2d(world, 1, 1))
    # the tensor interface on device data
    t = torch.arange(1000, device="cuda", dtype=torch.float32) * (rank + 1)
    out["t_ar"] = comm.all_reduce_tensor(t).cpu()
    g = torch.empty(world * 6, device="cuda", dtype=torch.bfloat16)
    out["t_ag"] = comm.all_gather_tensor(g, torch.full((6,), rank + 1.0, device="cuda").bfloat16()).float().cpu()
    b = torch.full((5,), float(rank), device="cuda")
    out["t_bc"] = comm.broadcast_tensor(b, 1).cpu()
    got = comm.exchange_neighbors_tensor(torch.full((3, 4), rank + 10.0, device="cuda"),
                                         MeshTorusHybrid.new_2d(world, 1, 1))
    out["t_x"] = [x.cpu() for x in got]
    out["status"] = int(comm.ctx.status())
    return out


@needs2
def test_device_communicator_matches_host_world_2gpu():
    """The device backend (NVLink peer-memory kernels) runs the reference's collective,
    point-to-point and neighbour-exchange cases with the host LocalWorld's results."""
    from comm_scenario import host_results
    from mtorus.core.topology import MeshTorusHybrid

    ref = host_results(2, MeshTorusHybrid.new_2d(2, 1, 1))
    got = run_dist(_device_comm_body, 2, backend="nccl")
    for r in range(2):
        for k, v in ref[r].items():
            assert got[r][k] == v, (r, k, got[r][k], v)
        assert got[r]["status"] == 0
        assert torch.equal(got[r]["t_ar"], torch.arange(1000, dtype=torch.float32) * 3)
        assert torch.equal(got[r]["t_ag"], torch.cat([torch.full((6,), 1.0), torch.full((6,), 2.0)]))
        assert torch.equal(got[r]["t_bc"], torch.full((5,), 1.0))
        # neighbours in +x, -x, +y, -y order: the other rank twice, then this rank twice
        want = [1 - r, 1 - r, r, r]
        assert [float(x[0, 0]) for x in got[r]["t_x"]] == [w + 10.0 for w in want]
