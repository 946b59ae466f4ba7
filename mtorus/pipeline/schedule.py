"""Pipeline schedules: GPipe and 1F1B.

Op lists come from the C++ builder (``mtorus._C.build_schedule``), which
reproduces crates/mt-pipeline/src/schedule/onef1b.rs:16-46 (warmup =
min(S-s-1, M) forwards, steady (F, B) pairs, cooldown backwards) and GPipe's
all-forwards-then-all-backwards order.

``GpipeSchedule.execute`` / ``OneF1BSchedule.execute`` are the reference's
single-process simulators (all stages in one thread, fixed ones(2x2) inputs
and gradients, FP8 stage transfer through ``PipelineComm``), kept for parity.
Real multi-rank execution is ``mtorus.pipeline.executor.DistributedPipelineExecutor``.
"""
from __future__ import annotations

import abc
from typing import List, Sequence

from .._ext import host as _host
from .communicator import PipelineComm
from .stage import PipelineStage, StageData

_C = _host()
ScheduleType = _C.ScheduleType
PipeOp = _C.PipeOp
build_schedule = _C.build_schedule
rank_program = _C.rank_program
simulate_schedule = _C.simulate_schedule
ideal_bubble_fraction = _C.ideal_bubble_fraction


class Schedule(abc.ABC):
    @abc.abstractmethod
    def execute(self, stages: List[PipelineStage], comms: Sequence[PipelineComm], num_microbatches: int) -> None: ...


def _ones22() -> StageData:
    return StageData([1.0] * 4, 2, 2)


class GpipeSchedule(Schedule):
    """All forwards, then all backwards (reference gpipe.rs:9-58)."""

    def execute(self, stages, comms, num_microbatches):
        S = len(stages)
        if S == 0:
            return
        inputs = [[] for _ in range(S)]
        for _ in range(num_microbatches):
            act = _ones22()
            for s, stage in enumerate(stages):
                inputs[s].append(act.clone())
                act = stage.forward(act)
                if s < S - 1:
                    comms[s].send_activations(act, s + 1)
                    act = comms[s + 1].recv_activations(s)
        for mb in range(num_microbatches):
            grad = _ones22()
            for s in range(S - 1, -1, -1):
                gin = stages[s].backward(inputs[s][mb].clone(), grad.clone())
                if s > 0:
                    comms[s].send_gradients(gin, s - 1)
                    grad = comms[s - 1].recv_gradients(s)


class OneF1BSchedule(Schedule):
    """Lock-step 1F1B ticks over the stages (reference onef1b.rs:50-111)."""

    @staticmethod
    def build_schedule(num_stages: int, num_microbatches: int):
        return build_schedule(ScheduleType.OneF1B, num_stages, num_microbatches)

    def execute(self, stages, comms, num_microbatches):
        S = len(stages)
        if S == 0:
            return
        sched = self.build_schedule(S, num_microbatches)
        stage_inputs = [[] for _ in range(S)]
        pending = [[] for _ in range(S)]
        idx = [0] * S
        max_ops = max(len(s) for s in sched)
        F = PipeOp.Kind.Forward
        while max_ops > 0:
            for s in range(S):
                if idx[s] >= len(sched[s]):
                    continue
                op = sched[s][idx[s]]
                if op.kind == F:
                    if s == 0:
                        inp = _ones22()
                    else:
                        pos = next(i for i, (m, _) in enumerate(pending[s]) if m == op.microbatch)
                        inp = pending[s].pop(pos)[1]
                    stage_inputs[s].append(inp.clone())
                    out = stages[s].forward(inp)
                    if s < S - 1:
                        comms[s].send_activations(out, s + 1)
                        pending[s + 1].append((op.microbatch, out))
                else:
                    gin = stages[s].backward(stage_inputs[s][op.microbatch].clone(), _ones22())
                    if s > 0:
                        comms[s].send_gradients(gin, s - 1)
                idx[s] += 1
            max_ops -= 1


class ScheduleKind(Schedule):
    """Enum dispatch over the two schedules (reference schedule/mod.rs:20-37)."""

    def __init__(self, inner: Schedule):
        self.inner = inner

    @staticmethod
    def Gpipe() -> "ScheduleKind":
        return ScheduleKind(GpipeSchedule())

    @staticmethod
    def OneF1B() -> "ScheduleKind":
        return ScheduleKind(OneF1BSchedule())

    def execute(self, stages, comms, num_microbatches):
        return self.inner.execute(stages, comms, num_microbatches)


__all__ = ["Schedule", "ScheduleKind", "GpipeSchedule", "OneF1BSchedule", "ScheduleType", "PipeOp",
           "build_schedule", "rank_program", "simulate_schedule", "ideal_bubble_fraction"]
