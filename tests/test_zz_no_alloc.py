"""The allocation-free LayerNorm backward C entry point.

Some callers cannot allocate device memory (an inference-engine plugin whose
enqueue must not call cudaMalloc, a server whose memory planner already owns
all of HBM).  ``mtorus_layernorm_bwd_noalloc`` serves them: it takes only
inputs and outputs and keeps its scratch in a fixed array inside the library.
This test calls it through its exported C symbol and compares it with the
regular torch-facing entry point on two calls in a row (the second call must
not see stale scratch from the first).
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _entry():
    from mtorus._ext import cuda

    lib = ctypes.CDLL(cuda().__file__)
    fn = lib.mtorus_layernorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return fn


def _case(rows, d, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, d, device="cuda", generator=g).bfloat16()
    dy = torch.randn(rows, d, device="cuda", generator=g).bfloat16()
    gamma = torch.randn(d, device="cuda", generator=g)
    beta = torch.randn(d, device="cuda", generator=g)
    return x, dy, gamma, beta


@pytest.mark.parametrize("rows,d", [(1024, 2048), (77, 256)])
def test_noalloc_matches_regular_entry_point_twice(rows, d):
    from mtorus.ops import kernels as K

    fn = _entry()
    stream = torch.cuda.current_stream()
    for call, seed in enumerate((11, 12)):
        x, dy, gamma, beta = _case(rows, d, seed)
        _, mean, rstd = K.layernorm_fwd(x, gamma, beta, 1e-5)
        dg_ref = torch.zeros(d, device="cuda")
        db_ref = torch.zeros(d, device="cuda")
        dx_ref = K.layernorm_bwd(dy, x, gamma, mean, rstd, dg_ref, db_ref, False)

        dx = torch.empty_like(x)
        dg = torch.full((d,), float("nan"), device="cuda")
        db = torch.full((d,), float("nan"), device="cuda")
        rc = fn(dy.data_ptr(), x.data_ptr(), gamma.data_ptr(), mean.data_ptr(), rstd.data_ptr(),
                dx.data_ptr(), dg.data_ptr(), db.data_ptr(), rows, d, 0, stream.cuda_stream)
        assert rc == 0, f"call {call}: return code {rc}"
        torch.cuda.synchronize()
        assert _rel(dx, dx_ref) < 2e-2, call
        assert _rel(dg, dg_ref) < 1e-2, call
        assert _rel(db, db_ref) < 1e-3, call


def test_noalloc_rejects_oversize_and_bad_args():
    fn = _entry()
    buf = torch.empty(8192 * 16, device="cuda", dtype=torch.float32)
    p = buf.data_ptr()
    s = torch.cuda.current_stream().cuda_stream
    assert fn(p, p, p, p, p, p, p, p, 4, 8192, 0, s) == -2  # d above the 4096 limit
    assert fn(p, p, p, p, p, p, p, p, 4, 12, 0, s) == -1    # d not a multiple of 8
    assert fn(None, p, p, p, p, p, p, p, 4, 256, 0, s) == -1
