"""FP8 casts around autograd: E4M3 for weights / activations forward, E5M2 for
gradients backward.

Reference: crates/mt-burn/src/autodiff_ext.rs.  ``gradient_cast_e5m2`` and
``weight_cast_e4m3`` quantise-dequantise with shape preserved.  The reference's
``GradientHook::cast_gradients_to_e5m2`` builds an all-ones shape (wrong for
numel > 1); here it preserves the shape like its ``_preserving_shape`` sibling.
``Fp8CastFn`` wires both casts into autograd, and ``install_fp8_grad_hooks``
casts every parameter gradient to E5M2 as it is produced.
"""
from __future__ import annotations

import torch

from ..core.precision import Fp8Format
from .fp8_ops import dequantize_tensor, quantize_tensor


def _fake_quant(x: torch.Tensor, fmt) -> torch.Tensor:
    q, s, _ = quantize_tensor(x, fmt)
    return dequantize_tensor(q, s).to(x.dtype).reshape(x.shape)


class GradientHook:
    @staticmethod
    def cast_gradients_to_e5m2(t: torch.Tensor) -> torch.Tensor:
        return _fake_quant(t, Fp8Format.E5M2)

    @staticmethod
    def cast_gradients_to_e5m2_preserving_shape(t: torch.Tensor) -> torch.Tensor:
        return _fake_quant(t, Fp8Format.E5M2)


class AutodiffExt:
    @staticmethod
    def gradient_cast_e5m2(grad: torch.Tensor) -> torch.Tensor:
        return _fake_quant(grad, Fp8Format.E5M2)

    @staticmethod
    def weight_cast_e4m3(weight: torch.Tensor) -> torch.Tensor:
        return _fake_quant(weight, Fp8Format.E4M3)


gradient_cast_e5m2 = AutodiffExt.gradient_cast_e5m2
weight_cast_e4m3 = AutodiffExt.weight_cast_e4m3


class Fp8CastFn(torch.autograd.Function):
    """Forward: E4M3 quantise-dequantise.  Backward: E5M2 quantise-dequantise of the gradient."""

    @staticmethod
    def forward(ctx, x):
        return _fake_quant(x, Fp8Format.E4M3)

    @staticmethod
    def backward(ctx, g):
        return _fake_quant(g, Fp8Format.E5M2)


def fp8_cast(x: torch.Tensor) -> torch.Tensor:
    return Fp8CastFn.apply(x)


def install_fp8_grad_hooks(module: torch.nn.Module):
    """Cast each parameter's gradient to E5M2 when it is computed; returns the hook handles."""
    return [p.register_hook(lambda g: _fake_quant(g, Fp8Format.E5M2)) for p in module.parameters() if p.requires_grad]


__all__ = ["GradientHook", "AutodiffExt", "gradient_cast_e5m2", "weight_cast_e4m3", "Fp8CastFn", "fp8_cast",
           "install_fp8_grad_hooks"]
