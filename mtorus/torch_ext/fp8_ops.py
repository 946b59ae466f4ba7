"""FP8 <-> torch tensor conversion.

Reference: crates/mt-burn/src/fp8_ops.rs (fp8_to_burn*, burn*_to_fp8).  Here the
conversions keep shapes explicitly (the reference's generic ``fp8_to_burn<D>``
invents a shape for D > 1) and quantise on the tensor's own device with
torch's float8 types: scale = format_max / amax (reference constants 416 /
49152), round-to-nearest-even, saturation to the largest finite value.

``quantize_tensor`` / ``dequantize_tensor`` are the device-side building blocks
(``DeviceFp8Tensor``: codes in a float8 tensor + an fp32 scale on device, no
host round trip).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

import torch

from ..core.precision import Fp8Format, Fp8Tensor, fp8_format_max, fp8_max_finite, from_fp8

_DT = {int(Fp8Format.E4M3): torch.float8_e4m3fn, int(Fp8Format.E5M2): torch.float8_e5m2}


def torch_dtype(fmt) -> torch.dtype:
    return _DT[int(fmt)]


def quantize_tensor(x: torch.Tensor, fmt, scale: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """-> (fp8 codes as a float8 tensor, fp32 scale [1], fp32 amax [1]); all on x's device."""
    xf = x.detach().float()
    amax = xf.abs().amax().reshape(1) if xf.numel() else torch.zeros(1, device=x.device)
    if scale is None:
        scale = torch.where(amax > 0, torch.full_like(amax, fp8_format_max(fmt)) / amax.clamp_min(1e-30),
                            torch.ones_like(amax))
    mf = fp8_max_finite(fmt)
    q = (xf * scale).clamp(-mf, mf).to(torch_dtype(fmt))
    return q, scale.reshape(1).float(), amax


def dequantize_tensor(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return q.float() / scale


@dataclass
class DeviceFp8Tensor:
    """Device-resident FP8 tensor: float8 codes, fp32 scale(s), amax history."""

    data: torch.Tensor
    format: object
    scale: torch.Tensor
    block_scales: Optional[torch.Tensor] = None
    block_size: Optional[int] = None
    amax_history: List[torch.Tensor] = field(default_factory=list)

    @staticmethod
    def quantize(x: torch.Tensor, fmt) -> "DeviceFp8Tensor":
        q, s, a = quantize_tensor(x, fmt)
        return DeviceFp8Tensor(q, fmt, s, amax_history=[a])

    def dequantize(self) -> torch.Tensor:
        if self.block_scales is not None:
            flat = self.data.float().reshape(-1)
            idx = torch.arange(flat.numel(), device=flat.device) // self.block_size
            return (flat / self.block_scales[idx]).reshape(self.data.shape)
        return dequantize_tensor(self.data, self.scale)

    def to_host(self) -> Fp8Tensor:
        t = Fp8Tensor(self.data.view(torch.uint8).reshape(-1).cpu().tolist(), self.format, float(self.scale.item()))
        if self.block_scales is not None:
            t.block_scales = self.block_scales.cpu().tolist()
            t.block_size = self.block_size
        t.amax_history = [float(a.item()) for a in self.amax_history]
        return t


def torch_to_fp8(t: torch.Tensor, fmt) -> Fp8Tensor:
    """Per-tensor quantisation into the host container (reference burn_to_fp8)."""
    q, s, a = quantize_tensor(t.reshape(-1), fmt)
    out = Fp8Tensor(q.view(torch.uint8).cpu().tolist(), fmt, float(s.item()))
    out.amax_history = [float(a.item())]
    return out


def torch_1d_to_fp8(t: torch.Tensor, fmt) -> Fp8Tensor:
    return torch_to_fp8(t.reshape(-1), fmt)


def torch_2d_to_fp8(t: torch.Tensor, fmt) -> Fp8Tensor:
    assert t.dim() == 2
    return torch_to_fp8(t, fmt)


def fp8_to_torch(t: Fp8Tensor, shape: Optional[Sequence[int]] = None, device=None) -> torch.Tensor:
    """Dequantise a host Fp8Tensor (per-tensor or per-block scales) into a float32 tensor."""
    v = torch.tensor(from_fp8(t), dtype=torch.float32, device=device)
    return v.reshape(tuple(shape)) if shape is not None else v


def fp8_to_torch_1d(t: Fp8Tensor, device=None) -> torch.Tensor:
    return fp8_to_torch(t, (len(t),), device)


def fp8_to_torch_2d(t: Fp8Tensor, rows: int, cols: int, device=None) -> torch.Tensor:
    if rows * cols != len(t):
        raise ValueError("rows * cols must equal the tensor length")
    return fp8_to_torch(t, (rows, cols), device)


__all__ = ["torch_dtype", "quantize_tensor", "dequantize_tensor", "DeviceFp8Tensor", "torch_to_fp8",
           "torch_1d_to_fp8", "torch_2d_to_fp8", "fp8_to_torch", "fp8_to_torch_1d", "fp8_to_torch_2d"]
