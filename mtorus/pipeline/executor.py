"""Pipeline executors.

``PipelineExecutor`` / ``PipelineConfig`` / ``ScheduleType`` mirror
crates/mt-pipeline/src/executor.rs: the executor runs the configured schedule
over in-process stages (the reference's simulation).

``DistributedPipelineExecutor`` is the real one: each rank owns one stage (a
torch module) and runs the per-rank program from the C++ schedule builder --
receive activations, forward, send, receive gradients, backward, send -- with
point-to-point transfers through ``torch.distributed`` (NCCL on GPUs, gloo on
CPU).  Sends are posted asynchronously so transfers overlap the next compute
op; receives for the next op are posted before the current compute runs.
Activation checkpointing (``CheckpointStrategy.Full``) keeps only the stage
input of each in-flight micro-batch and recomputes the forward in backward.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence

import torch
import torch.distributed as dist

from .checkpoint import CheckpointStrategy
from .communicator import PipelineComm
from .schedule import GpipeSchedule, OneF1BSchedule, PipeOp, ScheduleKind, ScheduleType, rank_program
from .stage import PipelineStage


@dataclass
class PipelineConfig:
    num_stages: int = 1
    num_microbatches: int = 1
    checkpoint_strategy: CheckpointStrategy = CheckpointStrategy.None_
    schedule_type: object = field(default_factory=lambda: ScheduleType.Gpipe)


class PipelineExecutor:
    def __init__(self, stages: List[PipelineStage], comm: Sequence[PipelineComm], config: PipelineConfig):
        self.stages = stages
        self.comm = list(comm)
        self.config = config
        self.schedule = ScheduleKind(GpipeSchedule() if config.schedule_type == ScheduleType.Gpipe
                                     else OneF1BSchedule())

    def run(self) -> None:
        self.schedule.execute(self.stages, self.comm, self.config.num_microbatches)

    def num_stages(self) -> int:
        return len(self.stages)


class DistributedPipelineExecutor:
    """One pipeline stage per rank over torch.distributed point-to-point.

    module      this rank's stage (torch.nn.Module); its forward takes the previous
                stage's activation (stage 0: the micro-batch input)
    stage_ranks global ranks of stages 0..S-1 (this rank must be one of them)
    loss_fn     last stage only: loss_fn(output, target) -> scalar; the executor
                divides it by the number of micro-batches
    act_shape   shape of the tensor exchanged between stages (per micro-batch)
    """

    def __init__(self, module: torch.nn.Module, stage_ranks: Sequence[int], schedule_type=ScheduleType.OneF1B,
                 num_microbatches: int = 1, checkpoint: CheckpointStrategy = CheckpointStrategy.None_,
                 loss_fn: Optional[Callable] = None, act_shape: Sequence[int] = (), act_dtype=torch.float32,
                 device=None, group=None, on_backward_done: Optional[Callable[[int], None]] = None):
        self.module = module
        self.stage_ranks = list(stage_ranks)
        self.S = len(self.stage_ranks)
        self.rank = dist.get_rank()
        self.stage = self.stage_ranks.index(self.rank)
        self.M = num_microbatches
        self.schedule_type = schedule_type
        self.checkpoint = checkpoint
        self.loss_fn = loss_fn
        self.act_shape = tuple(act_shape)
        self.act_dtype = act_dtype
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.group = group
        self.on_backward_done = on_backward_done
        self.program = rank_program(schedule_type, self.stage, self.S, self.M)
        self.is_first = self.stage == 0
        self.is_last = self.stage == self.S - 1

    def _peer(self, stage: int) -> int:
        return self.stage_ranks[stage]

    def _stage_forward(self, x):
        return self.module(x)

    def run(self, inputs: Optional[Sequence[torch.Tensor]] = None,
            targets: Optional[Sequence[torch.Tensor]] = None) -> List[float]:
        """Runs one step of the schedule; returns the per-micro-batch losses
        (last stage) and leaves parameter gradients accumulated in the module."""
        K = PipeOp.Kind
        stash_in: Dict[int, torch.Tensor] = {}
        stash_out: Dict[int, torch.Tensor] = {}
        recv_act: Dict[int, torch.Tensor] = {}
        recv_grad: Dict[int, torch.Tensor] = {}
        pending_sends = []
        losses: List[float] = []
        peak = 0
        for op in self.program:
            m = op.microbatch
            if op.kind == K.RecvAct:
                buf = torch.empty(self.act_shape, dtype=self.act_dtype, device=self.device)
                dist.recv(buf, self._peer(op.peer), group=self.group)
                recv_act[m] = buf
            elif op.kind == K.RecvGrad:
                buf = torch.empty(self.act_shape, dtype=self.act_dtype, device=self.device)
                dist.recv(buf, self._peer(op.peer), group=self.group)
                recv_grad[m] = buf
            elif op.kind == K.Forward:
                x = inputs[m] if self.is_first else recv_act.pop(m)
                if not self.is_first:
                    x.requires_grad_(True)
                stash_in[m] = x
                if self.checkpoint is CheckpointStrategy.Full:
                    with torch.no_grad():
                        y = self._stage_forward(x)
                else:
                    y = self._stage_forward(x)
                if self.is_last:
                    if self.checkpoint is CheckpointStrategy.Full:
                        stash_out[m] = None
                    else:
                        loss = self.loss_fn(y, targets[m]) / self.M
                        stash_out[m] = loss
                else:
                    stash_out[m] = y
                peak = max(peak, len(stash_in))
            elif op.kind == K.SendAct:
                y = stash_out[m]
                pending_sends.append(dist.isend(y.detach().contiguous(), self._peer(op.peer), group=self.group))
            elif op.kind == K.Backward:
                x = stash_in.pop(m)
                y = stash_out.pop(m)
                if self.checkpoint is CheckpointStrategy.Full:
                    x = x.detach().requires_grad_(not self.is_first)
                    with torch.enable_grad():
                        y = self._stage_forward(x)
                        if self.is_last:
                            y = self.loss_fn(y, targets[m]) / self.M
                if self.is_last:
                    losses.append(float(y.detach()) * self.M)
                    torch.autograd.backward(y)
                else:
                    torch.autograd.backward(y, recv_grad.pop(m))
                if self.on_backward_done is not None:
                    self.on_backward_done(m)
                stash_in[m] = x  # keep for SendGrad
            elif op.kind == K.SendGrad:
                x = stash_in.pop(m)
                pending_sends.append(dist.isend(x.grad.contiguous(), self._peer(op.peer), group=self.group))
            if len(pending_sends) > 8:
                pending_sends.pop(0).wait()
        for w in pending_sends:
            w.wait()
        stash_in.clear()
        self.peak_inflight = peak
        return losses


__all__ = ["PipelineConfig", "PipelineExecutor", "DistributedPipelineExecutor", "ScheduleType"]
