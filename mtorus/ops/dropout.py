"""Dropout for the fused GPT path, drawn from counter-based Philox4x32-10.

The reference GPT drops with p = 0.1 at five sites (examples/gpt-1b/src/
transformer.rs:77 attention probabilities, :108 the FFN hidden after GELU,
:148 / :154 the attention and FFN branch outputs before the residual adds;
model.rs:118 the embedding output).  Here each site's mask is drawn inside the
kernel that produces the tensor (the embedding kernel, the GEMM epilogues, the
attention kernel) and drawn again, from the same Philox counters, by the kernel
of the backward pass that needs it, so no mask is stored between the two.

Mask rule (``csrc/kernels/philox.cuh``): element e of site s is kept when the
16-bit uniform of its 8-element group e // 8 -- Philox4x32-10 with counter
(e // 8 low word, high word, s, 0) and the step's 64-bit key -- is at least
round(p * 65536); kept values are scaled by 1 / (1 - p).  The key lives in device
memory (``DropoutState.rng``) and ``DropoutState.advance()`` moves it to the next
step on the device, so a step captured in a CUDA graph draws fresh masks at every
replay.  ``keep_mask_ref`` restates the rule in NumPy (the test oracle).
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

SITE_ATTN_PROBS, SITE_ATTN_OUT, SITE_FFN_ACT, SITE_FFN_OUT = 0, 1, 2, 3
SITE_EMBED = 0xFFFF


def site_id(layer: int, role: int) -> int:
    """Dropout call-site id of ``role`` in transformer layer ``layer``."""
    return layer * 8 + role


def threshold16(p: float) -> int:
    return int(round(p * 65536.0))


_M0, _M1, _W0, _W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Vectorised Philox4x32-10 over uint64 NumPy arrays holding 32-bit values."""
    mask = np.uint64(0xFFFFFFFF)
    c0, c1, c2, c3 = (np.asarray(x, dtype=np.uint64) & mask for x in (c0, c1, c2, c3))
    k0, k1 = np.uint64(k0) & mask, np.uint64(k1) & mask
    for _ in range(10):
        p0 = np.uint64(_M0) * c0
        p1 = np.uint64(_M1) * c2
        hi0, lo0 = p0 >> np.uint64(32), p0 & mask
        hi1, lo1 = p1 >> np.uint64(32), p1 & mask
        c0, c1, c2, c3 = (hi1 ^ c1 ^ k0) & mask, lo1, (hi0 ^ c3 ^ k1) & mask, lo0
        k0 = (k0 + np.uint64(_W0)) & mask
        k1 = (k1 + np.uint64(_W1)) & mask
    return c0, c1, c2, c3


def keep_mask_ref(numel: int, seed: int, site: int, p: float) -> np.ndarray:
    """bool[numel]: the keep mask of the first ``numel`` elements of a site."""
    groups = (numel + 7) // 8
    g = np.arange(groups, dtype=np.uint64)
    words = philox4x32_10(g & np.uint64(0xFFFFFFFF), g >> np.uint64(32), np.full(groups, site, np.uint64),
                          np.zeros(groups, np.uint64), seed & 0xFFFFFFFF, seed >> 32)
    u = np.empty((groups, 8), dtype=np.uint64)
    for j in range(8):
        u[:, j] = (words[j >> 1] >> np.uint64((j & 1) * 16)) & np.uint64(0xFFFF)
    return (u >= np.uint64(threshold16(p))).reshape(-1)[:numel]


class DropoutState:
    """Per-model dropout probability and the device-resident Philox key of the step."""

    def __init__(self, p: float, device, seed: int = 0):
        if not 0.0 <= p < 1.0:
            raise ValueError("dropout probability must be in [0, 1)")
        self.p = float(p)
        self.thr16 = threshold16(p)
        self.scale = 1.0 / (1.0 - p)
        self.base_seed = int(seed)
        # {key low, key high, step low, step high} of the current step as int32 words
        # (read as uint32 by the kernels)
        self.rng = torch.zeros(4, dtype=torch.int32, device=device)
        self.set_step(0)

    def key(self, step: int) -> int:
        """64-bit Philox key of a step: a SplitMix64 mix of (base seed, step)."""
        z = (self.base_seed * 0x9E3779B97F4A7C15 + step + 1) & 0xFFFFFFFFFFFFFFFF
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
        return z ^ (z >> 31)

    def set_step(self, step: int) -> None:
        k = self.key(step)
        as_i32 = lambda v: v - (1 << 32) if v >= (1 << 31) else v  # noqa: E731
        words = [k & 0xFFFFFFFF, k >> 32, step & 0xFFFFFFFF, (step >> 32) & 0xFFFFFFFF]
        self.rng.copy_(torch.tensor([as_i32(w) for w in words], dtype=torch.int32))
        self.step = step

    def advance(self) -> None:
        """Next step's key, computed on the device (no host sync; capturable)."""
        from .._ext import cuda as _cuda

        if self.rng.is_cuda:
            b = self.base_seed & 0xFFFFFFFFFFFFFFFF
            _cuda().dropout_advance(self.rng, b - (1 << 64) if b >= (1 << 63) else b)
        else:
            self.set_step(self.step + 1)
            return
        self.step += 1

    def seed_host(self) -> int:
        lo, hi = (int(v) & 0xFFFFFFFF for v in self.rng.tolist()[:2])
        return lo | (hi << 32)

    micro = 0  # micro-batch index of the forward being run (set by the trainers)

    def args(self, site: int):
        """(rng, site, thr16, scale) for the kernels; the micro-batch index goes into the
        site word's high half, so every micro-batch of a step draws its own masks."""
        if not 0 <= site < (1 << 16):
            raise ValueError("dropout site ids are 16-bit")
        return self.rng, int(site) | ((int(self.micro) & 0xFFFF) << 16), self.thr16, self.scale

    def layer_args(self, layer: int, role: int):
        return self.args(site_id(layer, role))


def active(st: Optional["DropoutState"]) -> bool:
    return st is not None and st.p > 0.0


__all__ = ["DropoutState", "keep_mask_ref", "philox4x32_10", "site_id", "threshold16", "active",
           "SITE_ATTN_PROBS", "SITE_ATTN_OUT", "SITE_FFN_ACT", "SITE_FFN_OUT", "SITE_EMBED"]
