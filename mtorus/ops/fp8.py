"""Device FP8 with delayed scaling: quantisation kernels, the amax-history state,
and the FP8 GEMM entry point.

Recipe (the reference's MixedPrecisionConfig defaults, crates/mt-core/src/
precision/config.rs): E4M3 for weights and activations in the forward pass,
E5M2 for gradients in the backward pass, per-tensor scales from a DelayedScaling
amax history (crates/mt-core/src/precision/scaling.rs) with the reference's
format maxima (416 / 49152).  All scales live on the device: quantisation reads
the slot's current scale, folds max|x| into the slot's running amax, and one
kernel per step rolls every history ring and recomputes the scales.  The first
step, whose history is empty, measures each tensor's amax right before
quantising it ("current" scaling).

FP8 GEMMs run on tcgen05 kind::f8f6f4 with fp32 accumulation; the epilogue
multiplies by the two operands' inverse scales.
"""
from __future__ import annotations

import os
from typing import Dict, Optional, Tuple

import torch

from .._ext import cuda as _cuda

E4M3, E5M2 = 0, 1
# producers that write FP8 codes themselves (on by default; "0" selects the separate quantise pass)
_FUSE_LN = os.environ.get("MTORUS_FP8_FUSE_LN", "1") != "0"
_FUSE_GELU = os.environ.get("MTORUS_FP8_FUSE_GELU", "1") != "0"
FMT_MAX = {E4M3: 416.0, E5M2: 49152.0}  # reference format maxima (float8 crate MAX)


def quantize(x: torch.Tensor, fmt: int, scale: Optional[torch.Tensor] = None,
             amax: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16 -> fp8 codes (uint8), scaled by ``scale`` (device scalar); max|x| folds into ``amax``."""
    x = x.contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    _cuda().fp8_quantize(x, out, scale, amax, int(fmt))
    return out


def dequantize(q: torch.Tensor, inv_scale: torch.Tensor, fmt: int) -> torch.Tensor:
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    _cuda().fp8_dequantize(q.contiguous(), out, inv_scale, int(fmt))
    return out


def quantize_blocks(x: torch.Tensor, fmt: int, block_size: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-block quantisation (reference to_fp8_per_block) on device: codes + one fp32 scale per block."""
    x = x.contiguous().float()
    nb = (x.numel() + block_size - 1) // block_size
    out = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    scales = torch.empty(nb, dtype=torch.float32, device=x.device)
    _cuda().fp8_quantize_blocks(x, out, scales, int(block_size), FMT_MAX[fmt], int(fmt))
    return out, scales


def gemm_fp8_gelu8(a, a_fmt: int, b, b_fmt: int, pre: torch.Tensor, act8: torch.Tensor, act_scale: torch.Tensor,
                   act_amax: torch.Tensor, act_fmt: int, *, bias=None, alpha=None, alpha2=None):
    """FP8 GEMM whose epilogue stores the pre-activation (bf16, for dGELU) and
    GELU(pre) straight as FP8 codes of the next GEMM's input (scale ``act_scale``,
    max|GELU| folded into ``act_amax``)."""
    _cuda().gemm_fp8_act8(a, False, int(a_fmt), b, False, int(b_fmt), pre, bias, None, None, None, alpha, alpha2,
                          False, act8, act_scale, act_amax, int(act_fmt))
    return pre


def gemm_fp8(a, a_fmt: int, b, b_fmt: int, out=None, *, a_mn=False, b_mn=False, bias=None, residual=None,
             act=None, aux=None, alpha=None, alpha2=None, accumulate=False, out_dtype=torch.bfloat16):
    M = a.shape[1] if a_mn else a.shape[0]
    N = b.shape[1] if b_mn else b.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    _cuda().gemm_fp8(a, bool(a_mn), int(a_fmt), b, bool(b_mn), int(b_fmt), out, bias, residual, act, aux,
                     alpha, alpha2, bool(accumulate))
    return out


class NcclAmaxSync:
    """Cross-rank amax max for delayed scaling through one NCCL all-reduce (MAX) of
    the step's amax vector before the scales roll (the baseline of the fused path)."""

    def __init__(self, group=None):
        self.group = group

    def quantize(self, x, out, scale, amax, slot, fmt):
        quantize(x, fmt, scale, amax, out=out)

    def reduce(self, amax: torch.Tensor) -> None:
        import torch.distributed as dist

        dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=self.group)


class SymmAmaxSync:
    """The amax all-reduce fused into the quantise kernels.  The
    last block of each quantise launch stores the rank's running amax for that
    tensor role into every peer's table (symmetric memory, NVLink stores, tagged
    with the step's epoch, double-buffered by step parity); at the end of the step
    a flag barrier and one gather kernel take the max over ranks.  No collective
    library call and no extra pass over the data."""

    def __init__(self, device, capacity: int, group=None):
        from ..parallel.symm import SymmBuffer, SymmContext

        self.ctx = SymmContext(device, group, num_slots=4)
        self.me, self.world = self.ctx.rank, self.ctx.world
        self.cap = capacity
        self.table = SymmBuffer(2 * self.world * capacity, torch.int64, device, group)
        self.counters = torch.zeros(capacity, dtype=torch.int32, device=device)
        # stamps are 1 + the context's device step counter (advanced at the end of
        # every reduce, on the stream): graph replays publish with fresh stamps
        self.epoch = 1
        self.ep_ptr = self.ctx.ep_ptr
        self.table.barrier()

    def quantize(self, x, out, scale, amax, slot, fmt):
        _cuda().fp8_quantize_ar(x.contiguous(), out, scale, amax, self.counters[slot:slot + 1], self.table.ptrs,
                                self.me, self.cap, slot, self.epoch & 1, self.epoch, int(fmt), self.ep_ptr)

    def publish_args(self, slot: int):
        """(counter, table pointers, me, cap, slot, parity, epoch) for kernels that publish;
        pass ``ep_ptr=self.ep_ptr`` with them."""
        return (self.counters[slot:slot + 1], self.table.ptrs, self.me, self.cap, slot, self.epoch & 1, self.epoch)

    def reduce(self, amax: torch.Tensor) -> None:
        # roles whose codes a GEMM epilogue wrote were not published by a quantise
        # kernel: publish every used slot's running amax (the same value for the rest)
        _cuda().fp8_amax_publish(amax, self.table.ptrs, self.me, self.cap, self.epoch & 1, self.epoch, self.ep_ptr)
        # every rank has published this step's amaxes (its publishing kernels precede the barrier)
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 0, self.epoch, 24, self.ep_ptr)
        _cuda().fp8_amax_gather(self.table.tensor, amax, self.world, self.cap, self.epoch & 1, self.epoch,
                                self.ep_ptr)
        self.ctx.advance_epoch()


class Fp8State:
    """Amax histories, scales and inverse scales of every FP8 tensor role of a model."""

    def __init__(self, device, history: int = 16, capacity: int = 4096):
        self.device = torch.device(device)
        self.history = history
        self.names: Dict[str, int] = {}
        self.fmts = []
        self.cap = capacity
        d = self.device
        # fixed capacity: views of these buffers are captured by kernels and saved for backward
        self.hist = torch.zeros(capacity, history, device=d)
        self.amax = torch.zeros(capacity, device=d)
        self.scale = torch.ones(capacity, device=d)
        self.inv = torch.ones(capacity, device=d)
        self.fmax = torch.zeros(capacity, device=d)
        self.cursor = 0
        self.cursor_dev = torch.zeros(1, dtype=torch.int32, device=d)  # ring position, advanced on device
        self.first_step = True
        self._measured = set()  # slots whose first-step scale is already set
        self.sync = None  # cross-rank amax reduction (data parallel), see set_amax_sync
        self.recipe = "tensor"  # "mx": the block GEMMs run MXFP8 (set by GptModel.enable_fp8)

    def set_amax_sync(self, sync) -> None:
        """Make every amax the max over the data-parallel ranks (``NcclAmaxSync`` or
        ``SymmAmaxSync``); all ranks must quantise the same roles each step."""
        self.sync = sync

    def _quantize(self, x, fmt, s, out):
        sl = slice(s, s + 1)
        if self.sync is not None:
            if out is None:
                out = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
            self.sync.quantize(x, out, self.scale[sl], self.amax[sl], s, fmt)
            return out
        return quantize(x, fmt, self.scale[sl], self.amax[sl], out=out)

    def slot(self, name: str, fmt: int) -> int:
        s = self.names.get(name)
        if s is None:
            s = len(self.fmts)
            if s >= self.cap:
                raise RuntimeError(f"Fp8State capacity {self.cap} exceeded")
            self.names[name] = s
            self.fmts.append(fmt)
            self.fmax[s] = FMT_MAX[fmt]
        return s

    def quantize(self, x: torch.Tensor, name: str, fmt: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """-> (codes, inverse-scale view).  The inverse scale is the one this step used."""
        s = self.slot(name, fmt)
        sl = slice(s, s + 1)
        self._first_step_scale(x, s)
        q = self._quantize(x, fmt, s, None)
        # the inverse scale stays valid until end_step(), i.e. through this step's backward
        return q, self.inv[sl]

    def quantize_colsum(self, x: torch.Tensor, name: str, fmt: int, colsum: torch.Tensor,
                        accumulate: bool) -> Tuple[torch.Tensor, torch.Tensor]:
        """Quantise a 2-D bf16 gradient and (+)= its column sums (the bias gradient)
        into ``colsum`` in one pass over x -> (codes, inverse-scale view)."""
        s = self.slot(name, fmt)
        sl = slice(s, s + 1)
        self._first_step_scale(x, s)
        out = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
        if isinstance(self.sync, SymmAmaxSync):
            args = self.sync.publish_args(s)
        else:
            args = (None, [], 0, self.cap, s, 0, 0)
        ep = self.sync.ep_ptr if isinstance(self.sync, SymmAmaxSync) else 0
        _cuda().fp8_quantize_colsum(x.contiguous(), out, self.scale[sl], self.amax[sl], colsum, bool(accumulate),
                                    *args, int(fmt), ep)
        return out, self.inv[sl]

    def epilogue_slot(self, name: str, fmt: int):
        """(scale, amax, inverse scale) views for a producer kernel that writes the
        role's FP8 codes itself, or None when it cannot: the first step (scale not
        known yet).  Under ``SymmAmaxSync`` the role's amax is published with the
        rest at the end of the step."""
        if self.first_step or not _FUSE_GELU:
            return None
        s = self.slot(name, fmt)
        sl = slice(s, s + 1)
        return self.scale[sl], self.amax[sl], self.inv[sl]

    def layernorm_quantize(self, x2d: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float,
                           name: str, fmt: int):
        """LayerNorm(x) straight to FP8 codes of tensor role ``name`` ->
        (codes, inverse-scale view, mean, rstd).  The first step, whose scale is
        measured on the tensor itself, takes the unfused route (bf16 LN, then quantise)."""
        if self.first_step or not _FUSE_LN:
            from . import kernels as K

            h, mean, rstd = K.layernorm_fwd(x2d, gamma, beta, eps)
            q, inv = self.quantize(h, name, fmt)
            return q, inv, mean, rstd
        s = self.slot(name, fmt)
        sl = slice(s, s + 1)
        out = torch.empty(x2d.shape, dtype=torch.uint8, device=x2d.device)
        if isinstance(self.sync, SymmAmaxSync):
            args = self.sync.publish_args(s)
        else:
            args = (None, [], 0, self.cap, s, 0, 0)
        ep = self.sync.ep_ptr if isinstance(self.sync, SymmAmaxSync) else 0
        mean, rstd = _cuda().layernorm_fwd_fp8(x2d.contiguous(), gamma, beta, float(eps), out, self.scale[sl],
                                               self.amax[sl], int(fmt), *args, ep)
        return out, self.inv[sl], mean, rstd

    def quantize_into(self, x: torch.Tensor, name: str, fmt: int, out: torch.Tensor):
        s = self.slot(name, fmt)
        sl = slice(s, s + 1)
        self._first_step_scale(x, s)
        self._quantize(x, fmt, s, out)
        return out, self.inv[sl]

    def _first_step_scale(self, x: torch.Tensor, s: int) -> None:
        """First step (empty history): scale from the tensor's own amax, measured on
        its first use only -- later micro-batches of the step keep that scale, since
        earlier micro-batches' saved codes are dequantised with it in backward."""
        if not self.first_step or s in self._measured:
            return
        sl = slice(s, s + 1)
        _cuda().fp8_amax(x.contiguous(), self.amax[sl])
        _cuda().fp8_scaling_update(self.hist[sl], self.amax[sl], self.scale[sl], self.inv[sl],
                                   self.fmax[sl], self.cursor, True)
        self._measured.add(s)

    def end_step(self) -> None:
        """Roll all histories (delayed scaling): the next step's scales come from them."""
        n = len(self.fmts)
        if n and self.sync is not None:
            self.sync.reduce(self.amax[:n])
        if n:
            _cuda().fp8_scaling_update(self.hist[:n], self.amax[:n], self.scale[:n], self.inv[:n], self.fmax[:n],
                                       self.cursor, False, self.cursor_dev)
        self.cursor = (self.cursor + 1) % self.history  # host mirror (stale under graph replay)
        self.first_step = False

    def state_dict(self) -> dict:
        """Format, scale, amax history and cursor of every tensor role (the
        reference's DelayedScaling{amax_history, history_length, cursor} per role)."""
        n = len(self.fmts)
        return {"names": dict(self.names), "fmts": list(self.fmts), "hist": self.hist[:n].cpu(),
                "scale": self.scale[:n].cpu(), "inv": self.inv[:n].cpu(), "amax": self.amax[:n].cpu(),
                "cursor": int(self.cursor_dev), "history": self.history, "first_step": self.first_step,
                "measured": sorted(self._measured)}

    def load_state_dict(self, sd: dict) -> None:
        for name, fmt in zip(sorted(sd["names"], key=sd["names"].get), sd["fmts"]):
            self.slot(name, fmt)
        n = len(sd["fmts"])
        self.hist[:n] = sd["hist"].to(self.device)
        self.scale[:n] = sd["scale"].to(self.device)
        self.inv[:n] = sd["inv"].to(self.device) if "inv" in sd else 1.0 / self.scale[:n]
        if "amax" in sd:
            self.amax[:n] = sd["amax"].to(self.device)
        self.cursor = sd["cursor"]
        self.cursor_dev.fill_(int(sd["cursor"]))
        self.first_step = sd.get("first_step", False)
        self._measured = set(sd.get("measured", []))


__all__ = ["E4M3", "E5M2", "FMT_MAX", "quantize", "dequantize", "quantize_blocks", "gemm_fp8", "gemm_fp8_gelu8",
           "Fp8State",
           "NcclAmaxSync", "SymmAmaxSync"]
