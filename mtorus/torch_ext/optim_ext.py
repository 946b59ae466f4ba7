"""Optimizers that consume FP8 gradients.

Reference: crates/mt-burn/src/optim_ext.rs -- ``Fp8Optimizer::step_fp8`` (no
implementors in the reference), ``Fp8Gradients`` (ordered (id, values) list
with register / remove / len / is_empty), ``update_weight_fp8`` (SGD:
w - lr * dequant(g)), ``cast_to_fp8`` / ``cast_from_fp8``.

Implemented optimizers: ``Fp8Sgd`` (the reference update) and ``Fp8Adam``
(dequantise each E5M2 gradient on its device, then Adam; on a flat buffer of a
flattened model the fused device kernel ``FusedAdam`` does the same in one pass).
"""
from __future__ import annotations

import abc
from typing import Dict, List, Optional, Tuple

import torch

from ..core.precision import Fp8Tensor, from_fp8, to_fp8
from ..training.accumulator import ParamId, param_id
from .fp8_ops import DeviceFp8Tensor, fp8_to_torch


class Fp8Gradients:
    def __init__(self):
        self.grads: List[Tuple[ParamId, object]] = []

    def register(self, pid: ParamId, values) -> None:
        self.grads.append((pid, values))

    def remove(self, pid: ParamId):
        for i, (p, v) in enumerate(self.grads):
            if p == pid:
                self.grads.pop(i)
                return v
        return None

    def __len__(self) -> int:
        return len(self.grads)

    def len(self) -> int:
        return len(self.grads)

    def is_empty(self) -> bool:
        return not self.grads


def update_weight_fp8(weight: torch.Tensor, grad_fp8: Fp8Tensor, lr: float) -> torch.Tensor:
    g = fp8_to_torch(grad_fp8, weight.shape, weight.device).to(weight.dtype)
    return weight - lr * g


def cast_to_fp8(values, fmt) -> Fp8Tensor:
    return to_fp8([float(v) for v in values], fmt)


def cast_from_fp8(t: Fp8Tensor) -> List[float]:
    return from_fp8(t)


class Fp8Optimizer(abc.ABC):
    @abc.abstractmethod
    def step_fp8(self, lr: float, module: torch.nn.Module, grads: Fp8Gradients, config) -> torch.nn.Module: ...


def _dequant(g, like: torch.Tensor) -> torch.Tensor:
    if isinstance(g, DeviceFp8Tensor):
        return g.dequantize().reshape(like.shape).to(like.device, torch.float32)
    if isinstance(g, Fp8Tensor):
        return fp8_to_torch(g, like.shape, like.device)
    return torch.as_tensor(g, dtype=torch.float32, device=like.device).reshape(like.shape)


class Fp8Sgd(Fp8Optimizer):
    def step_fp8(self, lr, module, grads, config=None):
        with torch.no_grad():
            for p in module.parameters():
                g = grads.remove(param_id(p))
                if g is not None:
                    p.sub_(lr * _dequant(g, p))
        return module


class Fp8Adam(Fp8Optimizer):
    def __init__(self, betas=(0.9, 0.999), eps: float = 1e-5, weight_decay: float = 0.0):
        self.betas = betas
        self.eps = eps
        self.weight_decay = weight_decay
        self.state: Dict[ParamId, Tuple[torch.Tensor, torch.Tensor, int]] = {}

    def step_fp8(self, lr, module, grads, config=None):
        b1, b2 = self.betas
        with torch.no_grad():
            for p in module.parameters():
                pid = param_id(p)
                g = grads.remove(pid)
                if g is None:
                    continue
                g = _dequant(g, p)
                if self.weight_decay:
                    g = g + self.weight_decay * p
                m, v, t = self.state.get(pid, (torch.zeros_like(p), torch.zeros_like(p), 0))
                t += 1
                m.mul_(b1).add_(g, alpha=1 - b1)
                v.mul_(b2).addcmul_(g, g, value=1 - b2)
                denom = (v / (1 - b2 ** t)).sqrt_().add_(self.eps)
                p.addcdiv_(m, denom, value=-lr / (1 - b1 ** t))
                self.state[pid] = (m, v, t)
        return module


__all__ = ["Fp8Gradients", "update_weight_fp8", "cast_to_fp8", "cast_from_fp8", "Fp8Optimizer", "Fp8Sgd", "Fp8Adam"]
