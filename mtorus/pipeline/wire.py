"""FP8 wire format for pipeline-stage transfers.

The reference compresses the activations and gradients that cross a stage
boundary to FP8 before sending them (PipelineComm, crates/mt-pipeline/src/
communicator.rs:44-73; used by the schedules at schedule/gpipe.rs:33-36,49-52).
Its host frame (one fp32 scale for the whole tensor, 29-byte header) is kept as
the host codec (``mtorus.pipeline.communicator``); the device pipeline uses this
block-scaled form instead, which needs no amax pass before the encode and cannot
saturate:

    buffer = codes[numel] (uint8, E4M3 or E5M2) || scales[ceil(numel / 32)] (uint8)

with one power-of-two scale (UE8M0 byte, ``X + 127``) per 32 consecutive values,
X the smallest integer with ``amax <= fmax * 2**X`` (the MX block rule; fmax 448 /
57344), codes ``fp8(x * 2**-X)`` rounded to nearest even, and the NaN byte 255 for
a block holding a NaN / Inf.  1.03 bytes per value on the wire instead of 2 (bf16)
or 4 (fp32).

CUDA tensors go through the sm_100a codec kernels (``fp8_wire_encode`` /
``fp8_wire_decode``, one pass each); CPU tensors (gloo ranks) through the plain
PyTorch restatement below, which is also the oracle the kernels are tested
against.
"""
from __future__ import annotations

import torch

from .._ext import cuda as _cuda

E4M3, E5M2 = 0, 1
_FMAX = {E4M3: 448.0, E5M2: 57344.0}
_TORCH_FP8 = {E4M3: torch.float8_e4m3fn, E5M2: torch.float8_e5m2}


def wire_bytes(numel: int) -> int:
    """Bytes of the encoded buffer of ``numel`` values."""
    return numel + (numel + 31) // 32


def _block_exponent(amax: torch.Tensor, fmax: float) -> torch.Tensor:
    fbits = torch.tensor([fmax], dtype=torch.float32).view(torch.int32).item()
    ef, mf = (fbits >> 23) & 0xFF, fbits & 0x7FFFFF
    ua = amax.contiguous().view(torch.int32)
    x = ((ua >> 23) & 0xFF) - ef + ((ua & 0x7FFFFF) > mf).to(torch.int32)
    return torch.where(amax > 0, x.clamp(-127, 127), torch.zeros_like(x))


def encode_ref(x: torch.Tensor, fmt: int) -> torch.Tensor:
    """Plain-PyTorch encoder (any device)."""
    n = x.numel()
    nb = (n + 31) // 32
    flat = torch.zeros(nb * 32, dtype=torch.float32, device=x.device)
    flat[:n] = x.reshape(-1).float()
    xb = flat.view(nb, 32)
    finite = torch.isfinite(xb).all(-1)
    amax = torch.where(finite, xb.abs().amax(-1), torch.zeros(nb, device=x.device))
    X = _block_exponent(amax, _FMAX[fmt])
    inv = torch.ldexp(torch.ones_like(amax), (-X).float())
    codes = (xb * inv[:, None]).to(_TORCH_FP8[fmt]).view(torch.uint8).reshape(-1)[:n]
    sf = torch.where(finite, X + 127, torch.full_like(X, 255)).to(torch.uint8)
    return torch.cat([codes, sf])


def decode_ref(buf: torch.Tensor, shape, dtype: torch.dtype, fmt: int) -> torch.Tensor:
    n = 1
    for s in shape:
        n *= int(s)
    nb = (n + 31) // 32
    codes, sf = buf[:n], buf[n:n + nb].to(torch.int32)
    scale = torch.ldexp(torch.ones(nb, device=buf.device), (sf - 127).float())
    scale = torch.where(sf == 255, torch.full_like(scale, float("nan")), scale)
    vals = torch.zeros(nb * 32, dtype=torch.float32, device=buf.device)
    vals[:n] = codes.view(_TORCH_FP8[fmt]).float()
    return (vals.view(nb, 32) * scale[:, None]).reshape(-1)[:n].to(dtype).reshape(shape)


def encode(x: torch.Tensor, fmt: int = E4M3) -> torch.Tensor:
    """x (bf16 / fp32) -> uint8 wire buffer of ``wire_bytes(x.numel())`` bytes."""
    if not x.is_cuda:
        return encode_ref(x, fmt)
    x = x.contiguous()
    n = x.numel()
    buf = torch.empty(wire_bytes(n), dtype=torch.uint8, device=x.device)
    _cuda().fp8_wire_encode(x if x.dtype in (torch.bfloat16, torch.float32) else x.float(), buf[:n], buf[n:],
                            int(fmt))
    return buf


def decode(buf: torch.Tensor, shape, dtype: torch.dtype = torch.bfloat16, fmt: int = E4M3,
           out: torch.Tensor = None) -> torch.Tensor:
    """uint8 wire buffer -> tensor of ``shape`` / ``dtype``."""
    if not buf.is_cuda:
        return decode_ref(buf, shape, dtype, fmt)
    n = 1
    for s in shape:
        n *= int(s)
    if out is None:
        out = torch.empty(tuple(shape), dtype=dtype if dtype in (torch.bfloat16, torch.float32) else torch.float32,
                          device=buf.device)
    _cuda().fp8_wire_decode(buf[:n], buf[n:], out, int(fmt))
    return out if out.dtype == dtype else out.to(dtype)


__all__ = ["E4M3", "E5M2", "wire_bytes", "encode", "decode", "encode_ref", "decode_ref"]
