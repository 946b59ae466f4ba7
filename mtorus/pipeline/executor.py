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
Activation checkpointing: ``Full`` keeps only the stage input of each
in-flight micro-batch and recomputes the whole stage forward in backward;
``Selective`` splits the stage's segments at the midpoint (the reference's
split, crates/mt-pipeline/src/checkpoint.rs:43-60), keeps the activations of
the first half and the midpoint output, and recomputes only the second half in
backward (half of Full's recompute, about half of None's activation memory).
A stage of one segment has no midpoint, so Selective runs it as Full, like the
reference.

``wire="fp8"`` compresses every stage transfer the way the reference's
PipelineComm does (crates/mt-pipeline/src/communicator.rs:44-73): activations as
E4M3 and gradients as E5M2 by default, in the block-scaled wire format of
``mtorus.pipeline.wire`` (one power-of-two scale per 32 values, ~1.03 bytes per
value), encoded just before the send and decoded right after the receive.
"""
from __future__ import annotations

import os
import sys
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence

import torch
import torch.distributed as dist

from .checkpoint import CheckpointStrategy, checkpoint_module
from .communicator import PipelineComm
from .schedule import GpipeSchedule, OneF1BSchedule, PipeOp, ScheduleKind, ScheduleType, rank_program
from .stage import PipelineStage
from . import wire as W


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
    stage_fn    optional forward callable used instead of ``module(x)``
    wire        "native" (send act_dtype tensors) or "fp8" (block-scaled FP8 codes:
                ``wire_act_fmt`` for activations, ``wire_grad_fmt`` for gradients)
    stage_segments  optional list of callables whose composition is the stage
                forward (e.g. one per layer); ``Selective`` checkpointing splits
                it at the midpoint.  Default: the children of an
                ``nn.Sequential`` module, else the single stage forward
    pre_forward called as pre_forward(microbatch) before each forward (e.g. to select
                the micro-batch's dropout masks; a recomputing backward is preceded
                by pre_backward, which can do the same)
    pre_backward  called as pre_backward(microbatch, k) before the k-th backward of
                the step (k = 0 .. M-1), e.g. to switch gradient accumulation on
                after the first micro-batch or to arm the data-parallel reducer on
                the last one
    grad_group  process group for the backward (gradient) transfers; default
                ``group``.  With NCCL, activations and gradients between the same
                two ranks must travel on different communicators: one NCCL stream
                per rank pair would serialise a send of activations behind a
                receive of gradients and the two neighbours would wait on each
                other
    sync_losses True: ``run`` returns the per-micro-batch losses as floats (one
                host sync each); False: it returns the mean loss as a device
                scalar (last stage) without synchronising
    timed       record CUDA events around every forward / backward; after ``run``
                ``busy_ms`` / ``span_ms`` / ``bubble_fraction`` hold this rank's
                compute time, first-to-last op span and idle share of that span

    Receives for the next compute op are posted before the current one runs, so
    transfers overlap compute; sends are asynchronous.
    """

    def __init__(self, module: torch.nn.Module, stage_ranks: Sequence[int], schedule_type=ScheduleType.OneF1B,
                 num_microbatches: int = 1, checkpoint: CheckpointStrategy = CheckpointStrategy.None_,
                 loss_fn: Optional[Callable] = None, act_shape: Sequence[int] = (), act_dtype=torch.float32,
                 device=None, group=None, on_backward_done: Optional[Callable[[int], None]] = None,
                 stage_fn: Optional[Callable] = None, pre_backward: Optional[Callable[[int, int], None]] = None,
                 grad_group=None, sync_losses: bool = True, timed: bool = False,
                 stage_segments: Optional[Sequence[Callable]] = None, wire: str = "native",
                 wire_act_fmt: int = W.E4M3, wire_grad_fmt: int = W.E5M2,
                 pre_forward: Optional[Callable[[int], None]] = None):
        if wire not in ("native", "fp8"):
            raise ValueError(f"wire must be 'native' or 'fp8', not {wire!r}")
        self.wire = wire
        self.wire_fmt = {True: wire_act_fmt, False: wire_grad_fmt}  # keyed by "is activation"
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
        self.grad_group = grad_group if grad_group is not None else group
        self.on_backward_done = on_backward_done
        self.stage_fn = stage_fn
        if stage_segments is None and stage_fn is None and isinstance(module, torch.nn.Sequential):
            stage_segments = list(module.children())
        self.segments = list(stage_segments) if stage_segments else []
        if checkpoint not in (CheckpointStrategy.None_, CheckpointStrategy.Full, CheckpointStrategy.Selective):
            raise ValueError(f"unknown checkpoint strategy {checkpoint!r}")
        # Selective with fewer than two segments has no midpoint: the reference caches
        # the input and runs the stage, which is Full
        if checkpoint is CheckpointStrategy.Selective and len(self.segments) < 2:
            self.checkpoint = CheckpointStrategy.Full
        self.pre_backward = pre_backward
        self.pre_forward = pre_forward
        self.sync_losses = sync_losses
        self.timed = timed and self.device.type == "cuda"
        self.program = rank_program(schedule_type, self.stage, self.S, self.M)
        self.is_first = self.stage == 0
        self.is_last = self.stage == self.S - 1
        self.busy_ms = self.span_ms = self.bubble_fraction = None

    def _peer(self, stage: int) -> int:
        return self.stage_ranks[stage]

    def connect(self) -> None:
        """Sets up the NCCL point-to-point connections to both neighbours, on both
        groups, with one message of the real size in each direction.

        NCCL connects a peer lazily, inside the first send / receive to it, and that
        setup is a blocking host-side handshake with the peer.  If it first happened
        in the middle of the schedule (a receive posted ahead of a forward), the
        host would wait for a neighbour whose GPU may itself be waiting on a
        transfer this host has not launched yet.  Done once, here, before any
        transfer kernel runs, nothing later blocks the host.  The ops are the same
        unbatched send / receive calls as the schedule's (a batched call may get a
        communicator of its own), ordered as a chain that resolves from its end:
        every stage sends downstream first and then receives from upstream."""
        self._connected = True
        if self.S == 1:
            return
        buf_out = self._wire_buffer()
        buf_out.zero_()
        buf_in = torch.empty_like(buf_out)
        works = []
        for grp, nxt, prv in ((self.group, self.stage + 1, self.stage - 1),
                              (self.grad_group, self.stage - 1, self.stage + 1)):
            if 0 <= nxt < self.S:
                works.append(dist.isend(buf_out, self._peer(nxt), group=grp))
            if 0 <= prv < self.S:
                works.append(dist.irecv(buf_in, self._peer(prv), group=grp))
        for w in works:
            w.wait()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    def _stage_forward(self, x):
        return self.stage_fn(x) if self.stage_fn is not None else self.module(x)

    def _wire_buffer(self) -> torch.Tensor:
        """Receive buffer of one transfer in the wire format."""
        if self.wire == "fp8":
            n = 1
            for d in self.act_shape:
                n *= int(d)
            return torch.empty(W.wire_bytes(n), dtype=torch.uint8, device=self.device)
        return torch.empty(self.act_shape, dtype=self.act_dtype, device=self.device)

    def _to_wire(self, t: torch.Tensor, activation: bool) -> torch.Tensor:
        t = t.detach().contiguous()
        if self.wire == "fp8":
            return W.encode(t, self.wire_fmt[activation])
        return t

    def _from_wire(self, buf: torch.Tensor, activation: bool) -> torch.Tensor:
        if self.wire == "fp8":
            return W.decode(buf, self.act_shape, self.act_dtype, self.wire_fmt[activation])
        return buf

    def _selective_forward(self, x):
        """First half of the segments with their activations kept; the second half
        under ``checkpoint_module`` (only the midpoint output is kept, the second
        half's forward runs again inside backward)."""
        split = len(self.segments) // 2
        for seg in self.segments[:split]:
            x = seg(x)
        tail = self.segments[split:]

        def second_half(h):
            for seg in tail:
                h = seg(h)
            return h

        return checkpoint_module(second_half, x)

    def run(self, inputs: Optional[Sequence[torch.Tensor]] = None,
            targets: Optional[Sequence[torch.Tensor]] = None):
        """Runs one step of the schedule and leaves parameter gradients accumulated
        in the module.  Returns the per-micro-batch losses (``sync_losses``) or the
        mean loss as a device scalar (last stage; ``None`` elsewhere)."""
        if not getattr(self, "_connected", False) and self.device.type == "cuda":
            self.connect()
        K = PipeOp.Kind
        prog = self.program
        stash_in: Dict[int, torch.Tensor] = {}
        stash_out: Dict[int, torch.Tensor] = {}
        recv_act: Dict[int, torch.Tensor] = {}
        recv_grad: Dict[int, torch.Tensor] = {}
        posted: Dict[int, tuple] = {}
        pending_sends = []
        losses: List = []
        peak = 0
        n_bwd = 0
        events = []
        scan = 0

        def post_until(limit: int) -> None:
            nonlocal scan
            while scan < min(limit, len(prog)):
                op = prog[scan]
                if op.kind in (K.RecvAct, K.RecvGrad):
                    buf = self._wire_buffer()
                    grp = self.group if op.kind == K.RecvAct else self.grad_group
                    posted[scan] = (buf, dist.irecv(buf, self._peer(op.peer), group=grp))
                scan += 1

        compute_idx = [i for i, op in enumerate(prog) if op.kind in (K.Forward, K.Backward)]
        next_compute = {a: b for a, b in zip(compute_idx, compute_idx[1:] + [len(prog)])}

        trace = os.environ.get("MTORUS_PP_TRACE") == "1"
        for i, op in enumerate(prog):
            m = op.microbatch
            if trace:
                print(f"[pp rank {self.rank}] op {i} {op.kind} mb {m}", file=sys.stderr, flush=True)
            if op.kind in (K.RecvAct, K.RecvGrad):
                post_until(i + 1)
                buf, work = posted.pop(i)
                work.wait()
                (recv_act if op.kind == K.RecvAct else recv_grad)[m] = self._from_wire(buf, op.kind == K.RecvAct)
                continue
            if op.kind in (K.Forward, K.Backward):
                # receives needed by the next compute op go out before this one runs
                post_until(next_compute[i])
                if self.timed:
                    ev0 = torch.cuda.Event(enable_timing=True)
                    ev0.record()
            if op.kind == K.Forward:
                if self.pre_forward is not None:
                    self.pre_forward(m)
                x = inputs[m] if self.is_first else recv_act.pop(m)
                if not self.is_first:
                    x.requires_grad_(True)
                stash_in[m] = x
                if self.checkpoint is CheckpointStrategy.Full:
                    with torch.no_grad():
                        y = self._stage_forward(x)
                elif self.checkpoint is CheckpointStrategy.Selective:
                    y = self._selective_forward(x)
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
                y = self._to_wire(stash_out[m], True)
                pending_sends.append((dist.isend(y, self._peer(op.peer), group=self.group), y))
            elif op.kind == K.Backward:
                if self.pre_backward is not None:
                    self.pre_backward(m, n_bwd)
                n_bwd += 1
                x = stash_in.pop(m)
                y = stash_out.pop(m)
                if self.checkpoint is CheckpointStrategy.Full:
                    x = x.detach().requires_grad_(not self.is_first)
                    with torch.enable_grad():
                        y = self._stage_forward(x)
                        if self.is_last:
                            y = self.loss_fn(y, targets[m]) / self.M
                if self.is_last:
                    losses.append(y.detach())
                    torch.autograd.backward(y)
                else:
                    torch.autograd.backward(y, recv_grad.pop(m))
                del y
                if self.on_backward_done is not None:
                    self.on_backward_done(m)
                stash_in[m] = x  # keep for SendGrad
            elif op.kind == K.SendGrad:
                x = stash_in.pop(m)
                gx = self._to_wire(x.grad, False)
                pending_sends.append((dist.isend(gx, self._peer(op.peer), group=self.grad_group), gx))
            if op.kind in (K.Forward, K.Backward) and self.timed:
                ev1 = torch.cuda.Event(enable_timing=True)
                ev1.record()
                events.append((ev0, ev1))
            if len(pending_sends) > 8:
                pending_sends.pop(0)[0].wait()
        for w, _ in pending_sends:
            w.wait()
        stash_in.clear()
        self.peak_inflight = peak
        if self.timed and events:
            events[-1][1].synchronize()
            self.busy_ms = sum(a.elapsed_time(b) for a, b in events)
            self.span_ms = events[0][0].elapsed_time(events[-1][1])
            self.bubble_fraction = max(0.0, 1.0 - self.busy_ms / self.span_ms) if self.span_ms > 0 else 0.0
        if self.sync_losses:
            return [float(v) * self.M for v in losses]
        if not losses:
            return None
        return torch.stack(losses).sum()


__all__ = ["PipelineConfig", "PipelineExecutor", "DistributedPipelineExecutor", "ScheduleType"]
