"""Wiring of the opt-in E5M2 gradient transport in ``SymmBucketReducer``, checked on
the CPU with recording stand-ins for the symmetric buffers and kernels: every bucket
is encoded from its own fp32 range (byte offset 4 * start) into the code buffer at
element offset start and the scale buffer at block offset start / 32, then reduced
with the same bucket bounds, chunk length, flag slot and epoch (the context's device
step counter, advanced by begin_step) as the fp32 path; the
buckets launch in order as their parameters become ready."""
import contextlib

import pytest
import torch

from mtorus.parallel import symm


class _Buf:
    def __init__(self, numel, dtype, device=None, group=None, zero=True):
        self.tensor = torch.zeros(numel, dtype=dtype)
        self.ptrs = [self.tensor.data_ptr() + 1000 * r for r in range(2)]  # rank 1 is "me"
        self.ptrs[1] = self.tensor.data_ptr()
        self.mc = 0


class _Ctx:
    def __init__(self, device, group=None, num_slots=1024):
        self.flags = _Buf(num_slots * 8, torch.int32)
        self.rank, self.world, self.num_slots = 1, 2, num_slots
        self.ep_ptr = 4242
        self.advanced = 0

    def advance_epoch(self):
        self.advanced += 1


class _P:
    def __init__(self, off, n):
        self.flat_offset, self._n = off, n

    def numel(self):
        return self._n


class _Flat:
    symmetric = True
    device = torch.device("cpu")

    def __init__(self, sizes):
        self.params, off = [], 0
        for n in sizes:
            self.params.append(_P(off, n))
            off += (n + 63) // 64 * 64
        self.numel = off
        self.grad = torch.zeros(1, dtype=torch.float32)
        self.symm_grad = _Buf(self.numel, torch.float32)


class _Rec:
    calls = []

    def __getattr__(self, name):
        def f(*a):
            _Rec.calls.append((name, a))
        return f


@pytest.fixture
def fakes(monkeypatch):
    monkeypatch.setattr(symm, "SymmBuffer", _Buf)
    monkeypatch.setattr(symm, "SymmContext", _Ctx)
    monkeypatch.setattr(torch.cuda, "Stream", lambda *a, **k: type("S", (), {"wait_event": lambda s, e: None})())
    monkeypatch.setattr(torch.cuda, "Event", lambda *a, **k: type("E", (), {"record": lambda s, *x: None})())
    monkeypatch.setattr(torch.cuda, "stream", lambda s: contextlib.nullcontext())
    monkeypatch.setattr(symm, "_cuda", lambda: _Rec())
    _Rec.calls = []


def test_e5m2_transport_encodes_and_reduces_every_bucket(fakes):
    flat = _Flat([3000, 5000, 700, 9000])
    r = symm.SymmBucketReducer(flat, bucket_bytes=4 * 6000, ctas=8, reserve_sms=0, grad_fp8=True)
    r.state = torch.zeros(16)
    assert r.codes.tensor.numel() == flat.numel and r.gsf.tensor.numel() == flat.numel // 32
    r.begin_step()
    r.on_ready(list(reversed(flat.params)))  # backward order
    quant = [a for n, a in _Rec.calls if n == "dp_quant_e5m2"]
    reduce = [a for n, a in _Rec.calls if n == "symm_rs_bucket_e5m2"]
    assert len(quant) == len(reduce) == len(r.plan.ranges)
    gbase, cbase, sbase = (flat.symm_grad.tensor.data_ptr(), r.codes.tensor.data_ptr(), r.gsf.tensor.data_ptr())
    for b, ((s, e), q, rd) in enumerate(zip(r.plan.ranges, quant, reduce)):
        assert s % 64 == 0 and (e - s) % 32 == 0
        assert q == (gbase + 4 * s, cbase + s, sbase + s // 32, e - s)
        codes, sfs, flags, me, start, ln, clen, slot, epoch, st, ctas, inv_n, mine, ep = rd
        assert (codes, sfs) == (r.codes.ptrs, r.gsf.ptrs) and me == 1
        # host epoch 0 + the context's device step counter (advanced once by begin_step)
        assert (start, ln, clen, slot, epoch, ctas, inv_n, mine, ep) == (s, e - s, r.clen[b], b, 0, 8, 0.5, gbase,
                                                                         4242)
    assert r.ctx.advanced == 1
    assert not any(n in ("symm_rs_bucket", "symm_rs_bucket_mc") for n, _ in _Rec.calls)


def test_fp32_transport_stays_the_default(fakes, monkeypatch):
    monkeypatch.delenv("MTORUS_DP_GRAD_FP8", raising=False)
    flat = _Flat([3000, 5000])
    r = symm.SymmBucketReducer(flat, bucket_bytes=4 * 6000, ctas=8, reserve_sms=0)
    r.state = torch.zeros(16)
    assert not r.grad_fp8 and not hasattr(r, "codes")
    r.begin_step()
    r.on_ready(flat.params)
    names = [n for n, _ in _Rec.calls]
    assert "symm_rs_bucket" in names and "dp_quant_e5m2" not in names


@pytest.mark.parametrize("world", [2, 3, 8])
def test_rank_chunks_tile_every_bucket_once(fakes, monkeypatch, world):
    """The shard map the sharded Adam uses: over all ranks, the (flat offset, length)
    chunks cover every bucket exactly once; each rank's compact offsets are 8-aligned,
    ascending and non-overlapping, and its shard size is their padded total."""
    flat = _Flat([3000, 5000, 700, 9000, 64, 12345])
    cover = torch.zeros(flat.numel, dtype=torch.int32)
    for me in range(world):
        class Ctx(_Ctx):
            def __init__(self, *a, **k):
                super().__init__(*a, **k)
                self.rank, self.world = me, world

        monkeypatch.setattr(symm, "SymmContext", Ctx)
        r = symm.SymmBucketReducer(flat, bucket_bytes=4 * 6000, ctas=8, reserve_sms=0, grad_fp8=False)
        end = 0
        for off, ln, moff in r.ranges.tolist():
            cover[off:off + ln] += 1
            assert moff % 8 == 0 and moff >= end
            end = moff + (ln + 7) // 8 * 8
        assert r.shard_numel == end
    covered = torch.zeros(flat.numel, dtype=torch.bool)
    for s, e in symm.BucketPlan(flat, 4 * 6000).ranges:
        covered[s:e] = True
    assert bool((cover[covered] == 1).all()) and bool((cover[~covered] == 0).all())
