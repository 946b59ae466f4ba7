"""Failure detection on the GPU without a GPU fault: a kernel waits on a flag that
nothing sets, gives up after a short limit, reports a status code, and the
context stays usable.  A wait whose flag is already set completes without a
status."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives():
    from mtorus._ext import cuda as _cuda

    ext = _cuda()
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    ext.wait_flag(flag, 1, 300.0, status, 77, waited)  # nothing ever sets the flag
    torch.cuda.synchronize()
    assert int(status) == 77
    assert 300e6 <= int(waited) < 5e9
    # the context is intact: ordinary work runs and gives the right answer
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2


def test_bounded_wait_returns_when_flag_is_set():
    from mtorus._ext import cuda as _cuda

    ext = _cuda()
    flag = torch.ones(1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    ext.wait_flag(flag, 1, 1000.0, status, 78, waited)
    torch.cuda.synchronize()
    assert int(status) == 0 and int(waited) < 1e9
