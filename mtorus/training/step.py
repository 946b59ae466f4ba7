"""The training step: accumulate, overflow check, clip, warmup, loss scale.

Reference: crates/mt-training/src/step.rs.  ``train_step`` drains one
micro-batch's gradients into the accumulator; a non-finite norm halves the
dynamic loss scale, resets the accumulator and raises ``StepError.Overflow``;
once ``accumulation_steps`` micro-batches are in, it clips (if configured),
computes the warmup learning rate, grows the loss scale and advances the
global step.  As in the reference, the optimizer update itself is applied by
the caller.

The device-resident equivalent used by the fused path (norm, overflow, loss
scale, clip and Adam in three kernels, no host sync) is
``mtorus.training.fused_optim.FusedAdam``.
"""
from __future__ import annotations

import logging
import math
import time
from dataclasses import dataclass
from typing import Iterable, Sequence

import torch

from .accumulator import GradientAccumulator, GradientsParams, list_param_ids
from .config import TrainingConfig

log = logging.getLogger("mtorus.training")


@dataclass
class StepMetrics:
    loss: float
    learning_rate: float
    step: int
    overflow: bool
    grad_norm: float


@dataclass
class TrainingMetrics:
    avg_loss: float
    total_steps: int
    total_time_secs: float
    overflow_count: int


class StepError(Exception):
    pass


class _Overflow(StepError):
    def __init__(self):
        super().__init__("gradient overflow detected, skipping step")


class _ShapeMismatch(StepError):
    def __init__(self, msg: str):
        super().__init__(f"gradient shape mismatch: {msg}")


class _Internal(StepError):
    def __init__(self, msg: str):
        super().__init__(f"step error: {msg}")


StepError.Overflow = _Overflow
StepError.ShapeMismatch = _ShapeMismatch
StepError.Internal = _Internal


class TrainingError(Exception):
    pass


class _TrainStepError(TrainingError):
    def __init__(self, step: int, source: StepError):
        self.step = step
        self.source = source
        super().__init__(f"step error at step {step}: {source}")


class _EmptyDataloader(TrainingError):
    def __init__(self):
        super().__init__("dataloader is empty")


TrainingError.StepError = _TrainStepError
TrainingError.EmptyDataloader = _EmptyDataloader


class Counter:
    """Mutable integer (the reference passes ``&mut usize global_step``)."""

    def __init__(self, value: int = 0):
        self.value = value

    def __int__(self):
        return self.value

    def __eq__(self, o):
        return self.value == (o.value if isinstance(o, Counter) else o)


def compute_grad_norm(values) -> float:
    t = torch.as_tensor(values, dtype=torch.float32)
    return float(t.pow(2).sum().sqrt()) if t.numel() else 0.0


def clip_grad_norm(grads: torch.Tensor, max_norm: float) -> float:
    """Scales ``grads`` in place to norm ``max_norm`` when its norm exceeds it; returns the norm."""
    norm = float(grads.float().pow(2).sum().sqrt())
    if norm > max_norm and norm > 0.0:
        grads.mul_(max_norm / norm)
    return norm


def check_overflow_values(raw) -> tuple:
    """(global L2 norm, non-finite?) over a {param: grad} map."""
    sq = 0.0
    for v in raw.values():
        sq += float(torch.as_tensor(v, dtype=torch.float32).pow(2).sum())
    norm = math.sqrt(sq) if sq == sq and sq != math.inf else sq
    return norm, (math.isnan(norm) or math.isinf(norm))


def apply_clip_norm(acc: GradientAccumulator, max_norm: float) -> None:
    total = 0.0
    for v in acc.raw_grads().values():
        total += float(v.pow(2).sum())
    total = math.sqrt(total)
    if total > max_norm and total > 0.0:
        s = max_norm / total
        for v in acc.raw_grads_mut().values():
            v.mul_(s)


def warmup_lr(config: TrainingConfig, global_step: int) -> float:
    if config.warmup_steps > 0 and global_step < config.warmup_steps:
        return config.learning_rate * global_step / config.warmup_steps
    return config.learning_rate


def train_step(grads: GradientsParams, loss_value: float, config: TrainingConfig, accumulator: GradientAccumulator,
               loss_scaler, global_step: Counter, module: torch.nn.Module) -> StepMetrics:
    ids = list_param_ids(module)
    raw_norm = accumulator.drain_from(grads, ids)
    overflow = math.isnan(raw_norm) or math.isinf(raw_norm)
    if overflow:
        loss_scaler.update(True)
        log.debug("overflow detected, loss scaler halved to %s", loss_scaler.scale())
        accumulator.reset()
        raise StepError.Overflow()
    if accumulator.step_count() >= config.accumulation_steps:
        if config.clip_grad_norm > 0.0:
            apply_clip_norm(accumulator, config.clip_grad_norm)
        lr = warmup_lr(config, global_step.value)
        loss_scaler.update(False)
        global_step.value += 1
        m = StepMetrics(loss_value, lr, global_step.value, overflow, raw_norm)
        if config.log_interval and global_step.value % config.log_interval == 0:
            log.info("step %d: loss=%.6f, lr=%.2e, grad_norm=%.4f", m.step, m.loss, m.learning_rate, m.grad_norm)
        return m
    return StepMetrics(loss_value, config.learning_rate, global_step.value, overflow, raw_norm)


def training_loop(model, dataloader: Iterable, config: TrainingConfig) -> TrainingMetrics:
    """The reference's loop scaffold (step.rs:187-243): iterates the data, counting steps."""
    start = time.perf_counter()
    acc = GradientAccumulator()
    it = iter(dataloader)
    try:
        first = next(it)
    except StopIteration:
        raise TrainingError.EmptyDataloader()
    steps = 0
    for _batch in [first, *it]:
        acc.reset()
        steps += 1
    el = time.perf_counter() - start
    log.info("training loop completed: steps=%d, time=%.2fs, overflows=%d", steps, el, 0)
    return TrainingMetrics(0.0, steps, el, 0)


__all__ = ["StepMetrics", "TrainingMetrics", "StepError", "TrainingError", "Counter", "compute_grad_norm",
           "clip_grad_norm", "check_overflow_values", "apply_clip_norm", "train_step", "training_loop",
           "warmup_lr"]
