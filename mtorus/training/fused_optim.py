"""Device-resident fused optimizers over flat parameter buffers.

One optimizer step is three kernel launches and no host synchronisation:

1. ``grad_sumsq``  -- Σg² and a non-finite flag over the flat gradient buffer;
2. ``finalize``    -- one thread: overflow decision, dynamic loss-scale update
   (halve with floor 1 on overflow, double after ``growth_interval`` clean
   steps; crates/mt-core/src/precision/loss_scale.rs:34-51), global-norm clip
   factor (crates/mt-training/src/step.rs:61-98) and the unscale multiplier;
3. ``adam`` / ``sgd`` -- the update of the fp32 master weights, skipped on
   overflow, writing the bf16 compute copy in the same pass.

The state block ``state`` (fp32, 16 slots) is readable by the host at any time
without stalling the step (``stats()`` syncs only when called).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from ..ops import kernels as K

ST_SUMSQ, ST_NONFINITE, ST_SCALE, ST_GROWTH, ST_GRADMUL, ST_SKIP, ST_NORM, ST_STEP, ST_OVERFLOWS = range(9)


@dataclass
class DeviceLossScaleConfig:
    init_scale: float = 1.0
    dynamic: bool = False
    growth_interval: int = 2000


class FusedAdam:
    """Adam (burn-optim defaults: beta1 0.9, beta2 0.999, eps 1e-5) on flat buffers."""

    def __init__(self, flat, lr: float = 3e-4, betas=(0.9, 0.999), eps: float = 1e-5,
                 weight_decay: float = 0.0, max_grad_norm: float = 0.0,
                 loss_scale: Optional[DeviceLossScaleConfig] = None,
                 master: Optional[torch.Tensor] = None, grad: Optional[torch.Tensor] = None,
                 w16: Optional[torch.Tensor] = None):
        self.flat = flat
        self.master = flat.master if master is None else master
        self.grad = flat.grad if grad is None else grad
        self.w16 = (flat.w16 if flat is not None else None) if w16 is None else w16
        self.lr = lr
        self.betas = betas
        self.eps = eps
        self.weight_decay = weight_decay
        self.max_grad_norm = max_grad_norm
        self.ls = loss_scale or DeviceLossScaleConfig()
        dev = self.master.device
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.state = torch.zeros(16, dtype=torch.float32, device=dev)
        self.state[ST_SCALE] = self.ls.init_scale

    @property
    def loss_scale_tensor(self) -> torch.Tensor:
        """1-element device view of the current loss scale (multiplies the loss gradient)."""
        return self.state[ST_SCALE:ST_SCALE + 1]

    def accumulate_norm(self, grad: Optional[torch.Tensor] = None) -> None:
        K.grad_sumsq(self.grad if grad is None else grad, self.state)

    def finalize(self) -> None:
        K.optim_finalize(self.state, self.ls.dynamic, self.ls.growth_interval, self.max_grad_norm, True)

    def update(self, lr: Optional[float] = None) -> None:
        K.adam_step(self.master, self.m, self.v, self.grad, self.w16, self.state,
                    self.lr if lr is None else lr, self.betas[0], self.betas[1], self.eps, self.weight_decay)

    def step(self, lr: Optional[float] = None) -> None:
        self.accumulate_norm()
        self.finalize()
        self.update(lr)

    def stats(self) -> dict:
        s = self.state.tolist()
        return {"loss_scale": s[ST_SCALE], "grad_norm": s[ST_NORM], "skipped": s[ST_SKIP] > 0,
                "steps": int(s[ST_STEP]), "overflows": int(s[ST_OVERFLOWS]),
                "growth_counter": int(s[ST_GROWTH])}


class FusedSGD(FusedAdam):
    """w -= lr * g (reference update_weight_fp8, crates/mt-burn/src/optim_ext.rs:44-63)."""

    def __init__(self, flat, lr: float = 1e-2, **kw):
        super().__init__(flat, lr=lr, **kw)
        self.m = self.v = None

    def update(self, lr: Optional[float] = None) -> None:
        K.sgd_step(self.master, self.grad, self.w16, self.state, self.lr if lr is None else lr)
