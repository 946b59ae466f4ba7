"""Host logic of the weight all-gather fused into the GEMM (``GatheredOperand``),
checked on the CPU: the ``overlap`` schedule's shard order, the copy of each remote
shard into the local gathered buffer, the output-column slices of a K-major B and
the per-shard partial sums of a K-sharded (MN-major) B.

The device pieces are replaced by stand-ins with the same contracts: the copy
engine by a memmove between host addresses, CUDA streams and events by no-ops
(the stand-in copies complete at once), and the FP8 GEMM by a PyTorch product of
the decoded E4M3 codes.  The kernels themselves are covered by the 2-GPU test in
test_multigpu.py.
"""
import contextlib
import ctypes

import pytest
import torch

from mtorus.parallel import symm


class _Stream:
    def __init__(self, *a, **k):
        pass

    def wait_stream(self, other):
        pass

    def wait_event(self, ev):
        pass


class _Event:
    def record(self, stream=None):
        pass


class _Cuda:
    copies = []

    @staticmethod
    def copy_async(dst, src, nbytes):
        _Cuda.copies.append(nbytes)
        ctypes.memmove(dst, src, nbytes)


def _gemm_fp8_cpu(a, a_fmt, b, b_fmt, out=None, *, a_mn=False, b_mn=False, bias=None, residual=None, act=None,
                  aux=None, alpha=None, alpha2=None, accumulate=False, out_dtype=torch.bfloat16):
    A = a.view(torch.float8_e4m3fn).float()
    B = b.view(torch.float8_e4m3fn).float()
    A = A.t() if a_mn else A
    B = B if b_mn else B.t()  # [K, N]
    y = A @ B
    if alpha is not None:
        y = y * float(alpha)
    if bias is not None:
        y = y + bias
    if accumulate:
        out += y.to(out.dtype)
    else:
        out.copy_(y.to(out.dtype))
    return out


def _world(rows, cols, world, seed=0):
    """Per-rank 'symmetric' buffers holding only their own rows of a full code matrix."""
    g = torch.Generator().manual_seed(seed)
    full = (torch.randn(rows, cols, generator=g) * 0.5).to(torch.float8_e4m3fn).view(torch.uint8)
    per = (rows + world - 1) // world
    shard = (per + 127) // 128 * 128
    bufs = [torch.zeros(shard * world, cols, dtype=torch.uint8) for _ in range(world)]
    for p in range(world):
        lo, hi = min(rows, p * shard), min(rows, (p + 1) * shard)
        bufs[p][lo:hi] = full[lo:hi]
    return full, bufs, shard


def _operand(me, rows, cols, world, bufs, shard):
    op = symm.GatheredOperand.__new__(symm.GatheredOperand)
    op.me, op.world, op.rows, op.cols, op.shard_rows = me, world, rows, cols, shard
    op.full = bufs[me][:rows]
    op.lo, op.hi = op.shard_range(me)
    op.buf = type("B", (), {"ptrs": [b.data_ptr() for b in bufs]})()
    op._gathered, op._copy_stream = None, None
    return op


@pytest.fixture
def fake_device(monkeypatch):
    monkeypatch.setattr(symm, "_cuda", lambda: _Cuda)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a, **k: _Stream())
    monkeypatch.setattr(torch.cuda, "Stream", _Stream)
    monkeypatch.setattr(torch.cuda, "Event", _Event)
    monkeypatch.setattr(torch.cuda, "stream", lambda s: contextlib.nullcontext())
    import mtorus.ops.fp8 as F8

    monkeypatch.setattr(F8, "gemm_fp8", _gemm_fp8_cpu)
    _Cuda.copies = []
    yield


@pytest.mark.parametrize("world,me", [(2, 0), (2, 1), (4, 3)])
def test_overlap_kmajor_matches_full_product(fake_device, world, me):
    N, K, M = 640, 96, 48  # 640 rows over 4 ranks: shards of 256, the last one short
    full, bufs, shard = _world(N, K, world, seed=world + me)
    op = _operand(me, N, K, world, bufs, shard)
    a = (torch.randn(M, K) * 0.5).to(torch.float8_e4m3fn).view(torch.uint8)
    bias = torch.randn(N)
    out = torch.zeros(M, N)
    op.gemm(a, 0, 0, out, bias=bias, method="overlap", out_dtype=torch.float32)
    ref = _gemm_fp8_cpu(a, 0, full, 0, torch.zeros(M, N), bias=bias)
    assert torch.allclose(out, ref, rtol=1e-6, atol=1e-5)
    # every remote shard copied once, the own one never
    remote = sum(min(N, (p + 1) * shard) - min(N, p * shard) for p in range(world) if p != me)
    assert sum(_Cuda.copies) == remote * K


def test_overlap_ksharded_sums_partial_products(fake_device):
    world, me = 4, 1
    K, N, M = 512, 64, 40  # B stored [K, N], sharded along K in blocks of 128
    full, bufs, shard = _world(K, N, world, seed=7)
    op = _operand(me, K, N, world, bufs, shard)
    a = (torch.randn(M, K) * 0.5).to(torch.float8_e4m3fn).view(torch.uint8)
    out = torch.full((M, N), 3.0)  # accumulate=True adds onto what is there
    op.gemm(a, 0, 0, out, b_mn=True, accumulate=True, method="overlap")
    ref = 3.0 + _gemm_fp8_cpu(a, 0, full, 0, torch.zeros(M, N), b_mn=True)
    assert torch.allclose(out, ref, rtol=1e-5, atol=1e-4)
    with pytest.raises(ValueError):
        op.gemm(a, 0, 0, torch.zeros(M, N, dtype=torch.bfloat16), b_mn=True, method="overlap")


def test_auto_picks_direct_only_for_small_m(fake_device, monkeypatch):
    full, bufs, shard = _world(256, 64, 2)
    op = _operand(0, 256, 64, 2, bufs, shard)
    calls = []
    monkeypatch.setattr(op, "_gemm_overlap", lambda *a, **k: calls.append("overlap"))

    class _Direct(_Cuda):
        @staticmethod
        def gemm_fp8_gather_b(*a, **k):
            calls.append("direct")

    monkeypatch.setattr(symm, "_cuda", lambda: _Direct)
    x = torch.zeros(512, 64, dtype=torch.uint8)
    op.gemm(x, 0, 0, torch.zeros(512, 256))
    op.gemm(torch.zeros(513, 64, dtype=torch.uint8), 0, 0, torch.zeros(513, 256))
    assert calls == ["direct", "overlap"]
