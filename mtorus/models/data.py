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


__all__ = ["SyntheticDataLoader"]
