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


class DelayedCast:
    """One FP8 tensor role with delayed scaling: a ``DelayedScaling`` amax history
    (crates/mt-core/src/precision/scaling.rs) and a format.  ``cast(x)`` quantises
    with the scale from the history *before* x, then records max|x|; the first
    cast, whose history is empty, scales by x's own amax."""

    def __init__(self, fmt, history: int = 16):
        from ..core.precision import DelayedScaling

        self.fmt = fmt
        self.ds = DelayedScaling(history)
        self.used = False

    def cast(self, x: torch.Tensor) -> torch.Tensor:
        amax = float(x.detach().abs().max()) if x.numel() else 0.0
        if self.used:
            scale = self.ds.compute_scale(self.fmt)
            q, s, _ = quantize_tensor(x, self.fmt, torch.tensor([scale], device=x.device))
        else:
            q, s, _ = quantize_tensor(x, self.fmt)
            self.used = True
        self.ds.update(amax)
        return dequantize_tensor(q, s).to(x.dtype).reshape(x.shape)


class _DelayedCastFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, fwd: DelayedCast, bwd: DelayedCast):
        ctx.bwd = bwd
        return fwd.cast(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.bwd.cast(g), None, None


def enable_fp8_linears(module: torch.nn.Module, history: int = 16) -> int:
    """Run every Linear of ``module`` in (simulated) FP8 with delayed scaling: the
    input and the weight are cast to E4M3 in the forward pass, their gradients to
    E5M2 in the backward pass, each role with its own amax history of ``history``
    steps (the reference's recipe: MixedPrecisionConfig defaults,
    crates/mt-core/src/precision/config.rs).  Works on any device; this is the
    CPU / reference-semantics path -- the B200 path runs real FP8 GEMMs
    (``mtorus.ops.fp8``).  Returns the number of layers converted."""
    import torch.nn.functional as F

    n = 0
    for mod in module.modules():
        w = getattr(mod, "weight", None)
        if not isinstance(w, torch.nn.Parameter) or w.dim() != 2 or not hasattr(mod, "bias"):
            continue
        if isinstance(mod, torch.nn.Embedding) or type(mod).__name__ == "Embedding":
            continue
        roles = {k: DelayedCast(f, history) for k, f in
                 (("x", Fp8Format.E4M3), ("gx", Fp8Format.E5M2), ("w", Fp8Format.E4M3), ("gw", Fp8Format.E5M2))}
        mod.fp8_roles = roles

        def fwd(x, mod=mod, roles=roles):
            xq = _DelayedCastFn.apply(x, roles["x"], roles["gx"])
            wq = _DelayedCastFn.apply(mod.weight, roles["w"], roles["gw"])
            b = None if mod.bias is None else mod.bias.to(x.dtype)
            return F.linear(xq, wq.to(x.dtype), b)

        mod.forward = fwd
        n += 1
    return n


__all__ = ["GradientHook", "AutodiffExt", "gradient_cast_e5m2", "weight_cast_e4m3", "Fp8CastFn", "fp8_cast",
           "install_fp8_grad_hooks", "DelayedCast", "enable_fp8_linears"]
