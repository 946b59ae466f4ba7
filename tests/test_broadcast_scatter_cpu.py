"""Chunk arithmetic of the scatter + multicast broadcast
(``SymmCollectives.broadcast_scatter_nvls``), checked on the CPU with one thread per
rank: the device barrier becomes a ``threading.Barrier``, the copy engine a memmove,
and the multicast store (``multimem.st``) a write of the same bytes into every
rank's buffer.  Uneven last chunks, empty chunks (fewer bytes than ranks x 16) and
every root are covered; the kernels run in the 2-GPU test of test_multigpu.py."""
import ctypes
import threading

import pytest
import torch

from mtorus.parallel import symm

MC_BASE = 1 << 52  # stand-in multicast addresses: offsets from this base


class _Fabric:
    def __init__(self, n, nbytes):
        self.bufs = [torch.full((nbytes,), 255, dtype=torch.uint8) for _ in range(n)]
        self.barrier = threading.Barrier(n)

    def cuda(self):
        fab = self

        class C:
            @staticmethod
            def symm_barrier(flags, me, slot, epoch, code):
                fab.barrier.wait(timeout=10)

            @staticmethod
            def copy_async(dst, src, nbytes):
                ctypes.memmove(dst, src, nbytes)

            @staticmethod
            def symm_broadcast_mc(src, mc, nbytes, ctas):
                assert nbytes % 16 == 0 and (mc - MC_BASE) % 16 == 0
                for b in fab.bufs:
                    ctypes.memmove(b.data_ptr() + (mc - MC_BASE), src, nbytes)

        return C


def _collective(fab, me, n):
    c = symm.SymmCollectives.__new__(symm.SymmCollectives)
    c.me, c.world, c.epoch, c.ctas = me, n, 0, 128
    c.ctx = type("Ctx", (), {"flags": type("F", (), {"ptrs": []})()})()
    t = fab.bufs[me]
    c.buf = type("Buf", (), {"tensor": t, "ptrs": [b.data_ptr() for b in fab.bufs], "mc": MC_BASE})()
    return c


@pytest.mark.parametrize("n,nbytes", [(2, 1040), (4, 4096), (8, 48), (8, 16), (3, 1 << 16)])
def test_every_rank_ends_with_the_roots_bytes(monkeypatch, n, nbytes):
    for root in range(n):
        fab = _Fabric(n, nbytes)
        payload = torch.randint(0, 255, (nbytes,), dtype=torch.uint8)
        fab.bufs[root].copy_(payload)
        monkeypatch.setattr(symm, "_cuda", fab.cuda)
        errors = []

        def run(me):
            try:
                _collective(fab, me, n).broadcast_scatter_nvls(nbytes, root)
            except Exception as e:  # noqa: BLE001 - surfaced below
                errors.append(e)
                fab.barrier.abort()

        ts = [threading.Thread(target=run, args=(r,)) for r in range(n)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        assert not errors, errors
        for r in range(n):
            assert torch.equal(fab.bufs[r], payload), (root, r)


def test_rejects_sizes_off_the_16_byte_grain(monkeypatch):
    fab = _Fabric(2, 64)
    monkeypatch.setattr(symm, "_cuda", fab.cuda)
    with pytest.raises(ValueError):
        _collective(fab, 0, 2).broadcast_scatter_nvls(40, 0)
