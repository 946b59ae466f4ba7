"""Flat parameter / gradient buffers.

All parameters of a model are re-pointed into one fp32 master buffer, with a
bf16 compute copy (``p.w16``) and an fp32 gradient view (``p.main_grad``) at the
same offsets.  Groups of parameters listed together by the model (for example
the q/k/v projection weights) are laid out back to back so that one GEMM can
consume them as a single [3d, d] matrix.  Group starts are aligned to 256 bytes.

This layout is what the fused optimizer and the data-parallel bucket reducer
operate on: a bucket is a contiguous byte range of the flat buffers.
"""
from __future__ import annotations

from typing import Iterable, List, Sequence

import torch

_ALIGN = 64  # elements (256 B of fp32)


def _round_up(n: int, a: int) -> int:
    return (n + a - 1) // a * a


class FlatParams:
    def __init__(self, groups: Sequence[Sequence[torch.nn.Parameter]], device,
                 grad_dtype: torch.dtype = torch.float32, with_w16: bool = True,
                 symmetric: bool = False, group=None):
        seen = set()
        self.params: List[torch.nn.Parameter] = []
        self.groups: List[List[torch.nn.Parameter]] = []
        offsets = []
        off = 0
        for g in groups:
            g2 = [p for p in g if id(p) not in seen]
            if not g2:
                continue
            off = _round_up(off, _ALIGN)
            for p in g2:
                seen.add(id(p))
                self.params.append(p)
                offsets.append(off)
                off += p.numel()
            self.groups.append(g2)
        self.numel = _round_up(off, _ALIGN)
        self.offsets = offsets
        self.device = torch.device(device)
        self.master = torch.zeros(self.numel, dtype=torch.float32, device=self.device)
        self.symmetric = symmetric
        if symmetric:
            # gradients and bf16 weights are read / written by peers over NVLink
            from .symm import SymmBuffer

            self.symm_grad = SymmBuffer(self.numel, grad_dtype, self.device, group)
            self.symm_w16 = SymmBuffer(self.numel, torch.bfloat16, self.device, group)
            self.grad = self.symm_grad.tensor
            self.w16 = self.symm_w16.tensor
        else:
            self.grad = torch.zeros(self.numel, dtype=grad_dtype, device=self.device)
            self.w16 = torch.zeros(self.numel, dtype=torch.bfloat16, device=self.device) if with_w16 else None
        with torch.no_grad():
            for p, o in zip(self.params, offsets):
                n = p.numel()
                self.master[o:o + n].copy_(p.data.reshape(-1).to(self.device, torch.float32))
                p.data = self.master[o:o + n].view(p.shape)
                p.main_grad = self.grad[o:o + n].view(p.shape)
                p.flat_offset = o
                if self.w16 is not None:
                    p.w16 = self.w16[o:o + n].view(p.shape)
            if self.w16 is not None:
                self.w16.copy_(self.master)

    def sync_w16(self) -> None:
        """Refresh the bf16 compute copy from the fp32 master (after a load)."""
        if self.w16 is not None:
            with torch.no_grad():
                self.w16.copy_(self.master)

    def contiguous_view(self, params: Iterable[torch.nn.Parameter], which: str = "w16"):
        """Flat 1-D view spanning params that were laid out back to back."""
        ps = list(params)
        o0 = ps[0].flat_offset
        n = sum(p.numel() for p in ps)
        for a, b in zip(ps, ps[1:]):
            assert b.flat_offset == a.flat_offset + a.numel(), "params are not contiguous"
        buf = {"w16": self.w16, "master": self.master, "grad": self.grad}[which]
        return buf[o0:o0 + n]
