"""Synthetic token data.

Reference: examples/gpt-1b/src/synthetic_data.rs -- an iterator of (input,
target) [B, S] integer batches drawn uniformly from [0, vocab), with
``num_batches`` / ``current_batch`` / ``reset``.  The reference sets
target = input; ``shift=True`` gives next-token targets instead (draws S+1
tokens per row), which is what the benchmarks use.  Batches are seeded and can
be produced in pinned host memory for asynchronous H2D copies.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch


class SyntheticDataLoader:
    def __init__(self, batch_size: int, seq_len: int, vocab_size: int, num_batches: int, device=None,
                 seed: int = 0, shift: bool = False, pin_memory: bool = False):
        self.batch_size = batch_size
        self.seq_len = seq_len
        self.vocab_size = vocab_size
        self._num_batches = num_batches
        self.current = 0
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.seed = seed
        self.shift = shift
        self.pin_memory = pin_memory
        self._gen = torch.Generator().manual_seed(seed)

    def num_batches(self) -> int:
        return self._num_batches

    def current_batch(self) -> int:
        return self.current

    def reset(self) -> None:
        self.current = 0
        self._gen = torch.Generator().manual_seed(self.seed)

    def __iter__(self):
        return self

    def __next__(self) -> Tuple[torch.Tensor, torch.Tensor]:
        b = self.next()
        if b is None:
            raise StopIteration
        return b

    def next(self) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
        if self.current >= self._num_batches:
            return None
        self.current += 1
        n = self.seq_len + (1 if self.shift else 0)
        t = torch.randint(0, self.vocab_size, (self.batch_size, n), generator=self._gen, dtype=torch.long)
        if self.shift:
            inp, tgt = t[:, :-1].contiguous(), t[:, 1:].contiguous()
        else:
            inp, tgt = t, t.clone()
        if self.pin_memory and torch.cuda.is_available():
            inp, tgt = inp.pin_memory(), tgt.pin_memory()
        if self.device.type != "cpu":
            inp, tgt = inp.to(self.device, non_blocking=True), tgt.to(self.device, non_blocking=True)
        return inp, tgt


_MASK = (1 << 64) - 1


def _mix(z):
    """SplitMix64 finaliser on uint64 numpy arrays (the native loader's mixer)."""
    import numpy as np

    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def synthetic_batch_ref(seed: int, index: int, batch: int, seq_len: int, vocab: int, shift: bool):
    """Pure-Python/NumPy recomputation of batch ``index`` of ``NativeSyntheticDataLoader``."""
    import numpy as np

    n = seq_len + (1 if shift else 0)
    per = batch * n
    with np.errstate(over="ignore"):
        key = _mix(np.uint64((seed + 0x9E3779B97F4A7C15) & _MASK))
        ctr = np.uint64(index) * np.uint64(per) + np.arange(per, dtype=np.uint64)
        r = _mix(key ^ _mix(ctr))
    # (r * vocab) >> 64 without 128-bit integers: split r into 32-bit halves
    hi, lo = r >> np.uint64(32), r & np.uint64(0xFFFFFFFF)
    v = np.uint64(vocab)
    with np.errstate(over="ignore"):
        t = ((lo * v) >> np.uint64(32)) + hi * v
    tok = (t >> np.uint64(32)).astype(np.int64).reshape(batch, n)
    t = torch.from_numpy(tok)
    return (t[:, :-1].contiguous(), t[:, 1:].contiguous()) if shift else (t, t.clone())


class NativeSyntheticDataLoader:
    """``SyntheticDataLoader`` produced by the C++ runtime (``mtorus._C.TokenLoader``):
    worker threads generate batches ahead of the consumer into a ring, each batch a
    pure function of (seed, index), so ``seek(i)`` resumes a run exactly.  Batches are
    handed out in reusable (optionally pinned) host buffers -- copy or consume them
    before the next call -- and moved to ``device`` when one is given."""

    def __init__(self, batch_size: int, seq_len: int, vocab_size: int, num_batches: int, device=None,
                 seed: int = 0, shift: bool = False, pin_memory: bool = False, depth: int = 4, workers: int = 1):
        from .._ext import host as _host

        self._l = _host().TokenLoader(batch_size, seq_len, vocab_size, num_batches, seed, shift, depth, workers)
        self.batch_size, self.seq_len, self.vocab_size = batch_size, seq_len, vocab_size
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        pin = pin_memory and torch.cuda.is_available()
        self._inp = torch.empty((batch_size, seq_len), dtype=torch.long, pin_memory=pin)
        self._tgt = torch.empty((batch_size, seq_len), dtype=torch.long, pin_memory=pin)
        self._copied = None  # event after the last host-to-device copy out of the buffers

    def num_batches(self) -> int:
        return self._l.num_batches()

    def current_batch(self) -> int:
        return self._l.current_batch()

    def reset(self) -> None:
        self._l.reset()

    def seek(self, index: int) -> None:
        self._l.seek(index)

    def __iter__(self):
        return self

    def __next__(self):
        b = self.next()
        if b is None:
            raise StopIteration
        return b

    def next(self):
        if self._copied is not None:
            self._copied.synchronize()  # the previous asynchronous copy still reads the buffers
            self._copied = None
        if not self._l.next_into(self._inp.data_ptr(), self._tgt.data_ptr()):
            return None
        if self.device.type != "cpu":
            out = (self._inp.to(self.device, non_blocking=True), self._tgt.to(self.device, non_blocking=True))
            self._copied = torch.cuda.Event()
            self._copied.record()
            return out
        return self._inp, self._tgt


__all__ = ["SyntheticDataLoader", "NativeSyntheticDataLoader", "synthetic_batch_ref"]
