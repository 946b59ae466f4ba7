"""Activation checkpointing strategies.

Reference: crates/mt-pipeline/src/checkpoint.rs -- ``None`` runs the plain
forward, ``Full`` caches the stage input for recomputation, ``Selective`` runs
the first half of the layers, then the rest, and caches the input.  The torch
counterpart (``checkpoint_module``) recomputes a module's forward inside its
backward so only the module input is kept alive.
"""
from __future__ import annotations

import enum
from typing import List, Tuple

import torch

from .stage import PipelineStage, StageData, StageForward


class CheckpointStrategy(enum.Enum):
    Full = "Full"
    Selective = "Selective"
    None_ = "None"


# the reference spells the third variant ``None``
setattr(CheckpointStrategy, "NONE", CheckpointStrategy.None_)


class CheckpointHandle:
    def __init__(self, input: StageData):
        self.input = input


class ActivationCheckpoint:
    @staticmethod
    def save_input(input: StageData) -> CheckpointHandle:
        return CheckpointHandle(input.clone())

    @staticmethod
    def recompute_forward(handle: CheckpointHandle, layers: List[StageForward]) -> Tuple[StageData, StageData]:
        out = handle.input.clone()
        for layer in layers:
            out = layer.forward(out)
        return handle.input, out


def apply_checkpoint_forward(stage: PipelineStage, input: StageData, strategy: CheckpointStrategy) -> StageData:
    if strategy is CheckpointStrategy.None_:
        return stage.forward(input)
    if strategy is CheckpointStrategy.Full:
        stage.input_cache = input.clone()
        return stage.forward(input)
    if len(stage.layers) > 1:
        split = len(stage.layers) // 2
        out = input.clone()
        for layer in stage.layers[:split]:
            out = layer.forward(out)
        for layer in stage.layers[split:]:
            out = layer.forward(out)
        stage.input_cache = input.clone()
        return out
    stage.input_cache = input.clone()
    return stage.forward(input)


class _Recompute(torch.autograd.Function):
    @staticmethod
    def forward(ctx, fn, *inputs):
        ctx.fn = fn
        ctx.save_for_backward(*inputs)
        with torch.no_grad():
            return fn(*inputs)

    @staticmethod
    def backward(ctx, *grads):
        inputs = [x.detach().requires_grad_(x.requires_grad) for x in ctx.saved_tensors]
        with torch.enable_grad():
            out = ctx.fn(*inputs)
        outs = out if isinstance(out, tuple) else (out,)
        torch.autograd.backward(outs, grads)
        return (None,) + tuple(x.grad if x.requires_grad else None for x in inputs)


def checkpoint_module(fn, *inputs):
    """Run ``fn(*inputs)`` keeping only the inputs; the forward is recomputed in backward."""
    return _Recompute.apply(fn, *inputs)


__all__ = ["CheckpointStrategy", "CheckpointHandle", "ActivationCheckpoint", "apply_checkpoint_forward",
           "checkpoint_module"]
