"""FP8 mixed-precision primitives (C++ core codec + Python config types).

Reference: crates/mt-core/src/precision/{config,fp8_tensor,quantize,scaling,loss_scale}.rs.

* ``Fp8Format`` (E4M3 / E5M2), ``MasterFormat`` (Fp32 / Bf16), ``ScalingStrategy``
  (``Delayed(history_length)`` / ``Dynamic()``), ``MixedPrecisionConfig`` --
  defaults E4M3 forward, E5M2 backward, fp32 master, Delayed(1024).
* ``Fp8Tensor`` host container, ``to_fp8`` / ``to_fp8_with_scale`` /
  ``to_fp8_per_block`` / ``from_fp8``, ``Fp8Quantizer``.  Scale = format_max /
  amax with the reference's format maxima (416 for E4M3, 49152 for E5M2).
* ``DelayedScaling`` amax ring buffer, ``LossScaler`` (dynamic / static).

The device versions of these (block-scaled quantisation, the device amax ring,
the device loss scaler) live in ``mtorus.ops.fp8`` and ``mtorus.training.fused_optim``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Protocol, Sequence

from .._ext import host as _host

_C = _host()

Fp8Format = _C.Fp8Format
MasterFormat = _C.MasterFormat
LossScaleMode = _C.LossScaleMode
Fp8Tensor = _C.Fp8Tensor
DelayedScaling = _C.DelayedScaling
LossScaler = _C.LossScaler
fp8_format_max = _C.fp8_format_max
fp8_max_finite = _C.fp8_max_finite
fp8_encode = _C.fp8_encode
fp8_decode = _C.fp8_decode


def to_fp8(values: Sequence[float], fmt) -> Fp8Tensor:
    """Per-tensor quantisation: scale = fmt_max / amax (1 if amax == 0), history [amax]."""
    return _C.to_fp8(list(map(float, values)), fmt)


def to_fp8_with_scale(values: Sequence[float], fmt, scale: float) -> Fp8Tensor:
    return _C.to_fp8_with_scale(list(map(float, values)), fmt, float(scale))


def to_fp8_per_block(values: Sequence[float], fmt, block_size: int) -> Fp8Tensor:
    """Per-block scales (one fmt_max/amax per block); ``scale`` = first block's scale."""
    if block_size <= 0:
        raise ValueError("block_size must be > 0")
    return _C.to_fp8_per_block(list(map(float, values)), fmt, int(block_size))


def from_fp8(t: Fp8Tensor) -> List[float]:
    return _C.from_fp8(t)


class Quantize(Protocol):
    @staticmethod
    def to_fp8(values: Sequence[float], fmt) -> Fp8Tensor: ...

    @staticmethod
    def from_fp8(t: Fp8Tensor) -> List[float]: ...


class Fp8Quantizer:
    """The reference's ``Quantize`` implementation (quantize.rs:12-52)."""

    @staticmethod
    def to_fp8(values: Sequence[float], fmt) -> Fp8Tensor:
        return to_fp8(values, fmt)

    @staticmethod
    def from_fp8(t: Fp8Tensor) -> List[float]:
        return from_fp8(t)


class ScalingStrategy:
    """``Delayed { history_length }`` or ``Dynamic`` (config.rs:14-18)."""

    @dataclass(frozen=True)
    class Delayed:
        history_length: int = 1024

    @dataclass(frozen=True)
    class Dynamic:
        pass


@dataclass
class MixedPrecisionConfig:
    forward_format: object = field(default_factory=lambda: Fp8Format.E4M3)
    backward_format: object = field(default_factory=lambda: Fp8Format.E5M2)
    master_format: object = field(default_factory=lambda: MasterFormat.Fp32)
    scaling_strategy: object = field(default_factory=lambda: ScalingStrategy.Delayed(1024))

    # serde-style externally tagged encoding (TOML / dict)
    def to_dict(self) -> dict:
        s = self.scaling_strategy
        strat = ({"Delayed": {"history_length": s.history_length}}
                 if isinstance(s, ScalingStrategy.Delayed) else "Dynamic")
        return {"forward_format": self.forward_format.name, "backward_format": self.backward_format.name,
                "master_format": self.master_format.name, "scaling_strategy": strat}

    @staticmethod
    def from_dict(d: dict) -> "MixedPrecisionConfig":
        s = d.get("scaling_strategy", {"Delayed": {"history_length": 1024}})
        if s == "Dynamic" or (isinstance(s, dict) and "Dynamic" in s):
            strat = ScalingStrategy.Dynamic()
        else:
            strat = ScalingStrategy.Delayed(int(s["Delayed"]["history_length"]))
        return MixedPrecisionConfig(
            forward_format=getattr(Fp8Format, d.get("forward_format", "E4M3")),
            backward_format=getattr(Fp8Format, d.get("backward_format", "E5M2")),
            master_format=getattr(MasterFormat, d.get("master_format", "Fp32")),
            scaling_strategy=strat)


__all__ = [
    "Fp8Format", "MasterFormat", "ScalingStrategy", "MixedPrecisionConfig", "Fp8Tensor", "LossScaleMode",
    "LossScaler", "DelayedScaling", "Fp8Quantizer", "Quantize", "to_fp8", "from_fp8", "to_fp8_with_scale",
    "to_fp8_per_block", "fp8_format_max", "fp8_max_finite", "fp8_encode", "fp8_decode",
]
