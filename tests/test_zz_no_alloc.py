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


def _call(fn, x, dy, gamma, mean, rstd, dx, dg, db, accumulate):
    rows, d = x.shape
    return fn(dy.data_ptr(), x.data_ptr(), gamma.data_ptr(), mean.data_ptr(), rstd.data_ptr(),
              dx.data_ptr(), dg.data_ptr(), db.data_ptr(), rows, d, int(accumulate),
              torch.cuda.current_stream().cuda_stream)


def test_noalloc_after_regular_call_that_lowered_the_smem_limit():
    """A regular call with d = 2056 sets the 16-chunk kernel's shared-memory limit to
    its own ~64 KiB; a later allocation-free call with d = 4096 needs 128 KiB of it."""
    from mtorus.ops import kernels as K

    fn = _entry()
    x, dy, gamma, beta = _case(300, 2056, 21)
    _, mean, rstd = K.layernorm_fwd(x, gamma, beta, 1e-5)
    K.layernorm_bwd(dy, x, gamma, mean, rstd, torch.zeros(2056, device="cuda"),
                    torch.zeros(2056, device="cuda"), False)
    x, dy, gamma, beta = _case(300, 4096, 22)
    _, mean, rstd = K.layernorm_fwd(x, gamma, beta, 1e-5)
    dg_ref, db_ref = torch.zeros(4096, device="cuda"), torch.zeros(4096, device="cuda")
    dx_ref = K.layernorm_bwd(dy, x, gamma, mean, rstd, dg_ref, db_ref, False)
    dx = torch.empty_like(x)
    dg = torch.full((4096,), float("nan"), device="cuda")
    db = torch.full((4096,), float("nan"), device="cuda")
    assert _call(fn, x, dy, gamma, mean, rstd, dx, dg, db, 0) == 0
    torch.cuda.synchronize()
    assert _rel(dx, dx_ref) < 2e-2
    assert _rel(dg, dg_ref) < 1e-2
    assert _rel(db, db_ref) < 1e-3


def test_noalloc_accumulate_adds_to_existing_gradients():
    from mtorus.ops import kernels as K

    fn = _entry()
    rows, d = 513, 1024
    x, dy, gamma, beta = _case(rows, d, 31)
    _, mean, rstd = K.layernorm_fwd(x, gamma, beta, 1e-5)
    g0 = torch.Generator(device="cuda").manual_seed(32)
    dg0 = torch.randn(d, device="cuda", generator=g0)
    db0 = torch.randn(d, device="cuda", generator=g0)
    dg_ref, db_ref = dg0.clone(), db0.clone()
    dx_ref = K.layernorm_bwd(dy, x, gamma, mean, rstd, dg_ref, db_ref, True)
    dx = torch.empty_like(x)
    dg, db = dg0.clone(), db0.clone()
    assert _call(fn, x, dy, gamma, mean, rstd, dx, dg, db, 1) == 0
    torch.cuda.synchronize()
    assert _rel(dx, dx_ref) < 2e-2
    assert _rel(dg, dg_ref) < 1e-2
    assert _rel(db, db_ref) < 1e-3


def test_noalloc_rejects_oversize_and_bad_args():
    fn = _entry()
    buf = torch.empty(8192 * 16, device="cuda", dtype=torch.float32)
    p = buf.data_ptr()
    s = torch.cuda.current_stream().cuda_stream
    assert fn(p, p, p, p, p, p, p, p, 4, 8192, 0, s) == -2  # d above the 4096 limit
    assert fn(p, p, p, p, p, p, p, p, 4, 12, 0, s) == -1    # d not a multiple of 8
    assert fn(None, p, p, p, p, p, p, p, 4, 256, 0, s) == -1
