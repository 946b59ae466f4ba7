"""PipelineTrainer: GPT training with data x pipeline parallelism on the fused path.

The world of ``dp * pp`` ranks (one per GPU) is laid out as ``dp`` pipeline
replicas of ``pp`` consecutive ranks: rank = replica * pp + stage.  Each rank
builds only its stage of the model (``GptModel(layers=..., embed=..., head=...)``;
contiguous layer ranges as in the reference's crates/mt-burn/src/module_ext.rs:40-79,
balanced by FLOPs with the LM head counted (``balanced_split``) or ``split_evenly``),
flattens it into its own fp32 master /
bf16 / fp32-grad buffers and runs:

1. the per-rank GPipe or 1F1B program from the schedule builder
   (``DistributedPipelineExecutor``; reference crates/mt-pipeline/src/schedule/
   gpipe.rs, onef1b.rs) with NCCL point-to-point activations / gradients,
   activations on one process group and gradients on another so that the two
   directions between neighbours never share an NCCL stream;
2. optional activation checkpointing per stage: Full (stage input kept, forward
   recomputed in backward) or Selective (the second half of the stage's blocks
   recomputed from the midpoint output); reference
   crates/mt-pipeline/src/checkpoint.rs;
3. gradient accumulation over the micro-batches straight into ``main_grad``
   (the first backward overwrites, the rest add, in the wgrad GEMM epilogues);
4. during the last micro-batch's backward, the data-parallel gradient reduction
   over the ranks that hold the same stage, overlapped with that backward: NCCL
   bucket all-reduces (``dp="nccl"``) or the fused NVLink path (``dp="symm"``:
   per-bucket reduce-scatter kernels over symmetric memory with the norm /
   overflow partials fused, then the sharded Adam that stores the new weights
   into every peer, and the delayed-scaling amax all-reduce fused into the FP8
   quantise kernels);
5. the fused device optimizer, with the gradient-norm / overflow statistics
   summed over the pipeline so that every stage takes the same skip / clip /
   loss-scale decision (reference crates/mt-training/src/step.rs:114-180).

Stage placement: on one NVSwitch node every GPU pair is one NVLink hop, so
consecutive ranks per pipeline is already the topology-aware placement
(``topology_aware_placement`` maps stages to torus nodes across nodes).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from ..models.gpt import GptConfig, GptModel
from ..ops.fused import FusedGradState
from ..pipeline.checkpoint import CheckpointStrategy
from ..pipeline.executor import DistributedPipelineExecutor
from ..pipeline.schedule import ScheduleType, ideal_bubble_fraction
from ..torch_ext.module_ext import split_evenly
from .fused_optim import ST_NONFINITE, ST_SUMSQ, DeviceLossScaleConfig, FusedAdam


def stage_costs(config: GptConfig, seq_len: Optional[int] = None):
    """Forward FLOPs per token of each transformer layer and of the LM head + loss."""
    S = seq_len or config.max_seq_len
    d, f, V = config.d_model, config.d_ff, config.vocab_size
    layer = 2.0 * (4 * d * d + 2 * d * f) + 2.0 * S * d  # GEMMs + causal attention
    head = 2.0 * d * V + 8.0 * V  # LM head GEMM + softmax cross-entropy
    return layer, head


def balanced_split(config: GptConfig, pp: int, seq_len: Optional[int] = None) -> List[tuple]:
    """Contiguous layer ranges (lo, hi) for ``pp`` stages that minimise the slowest
    stage, counting the LM head on the last stage (for GPT-1B it costs about two
    layers).  Every stage gets at least one layer.  ``split_evenly`` (the reference's
    rule) ignores the head, which leaves the last stage the bottleneck of the
    schedule."""
    L = config.num_layers
    if pp < 1 or pp > L:
        raise ValueError(f"cannot split {L} layers into {pp} stages")
    layer, head = stage_costs(config, seq_len)
    INF = float("inf")
    # best[s][i]: min over splits of layers i..L-1 into stages s..pp-1 of the max stage cost
    best = [[INF] * (L + 1) for _ in range(pp + 1)]
    cut = [[0] * (L + 1) for _ in range(pp + 1)]
    best[pp][L] = 0.0
    for s in range(pp - 1, -1, -1):
        for i in range(L - 1, -1, -1):
            for j in range(i + 1, L - (pp - 1 - s) + 1):
                c = (j - i) * layer + (head if s == pp - 1 else 0.0)
                if s == pp - 1 and j != L:
                    continue
                v = max(c, best[s + 1][j])
                if v < best[s][i]:
                    best[s][i], cut[s][i] = v, j
    out, i = [], 0
    for s in range(pp):
        j = cut[s][i]
        out.append((i, j))
        i = j
    return out


@dataclass
class PipelineLayout:
    """Rank layout of a dp x pp job: ``stage_ranks[r]`` are the ranks of replica r
    (stage order); ``dp_ranks[s]`` the ranks that hold stage s."""

    dp: int
    pp: int
    stage_ranks: List[List[int]] = field(default_factory=list)
    dp_ranks: List[List[int]] = field(default_factory=list)

    def __post_init__(self):
        self.stage_ranks = [[r * self.pp + s for s in range(self.pp)] for r in range(self.dp)]
        self.dp_ranks = [[r * self.pp + s for r in range(self.dp)] for s in range(self.pp)]

    def coords(self, rank: int):
        """-> (replica, stage)."""
        return divmod(rank, self.pp)


class PipelineTrainer:
    def __init__(self, config: GptConfig, pp: int, dp: int = 1, schedule=ScheduleType.OneF1B,
                 num_microbatches: int = 8, micro_batch: int = 1, seq_len: Optional[int] = None,
                 checkpoint: CheckpointStrategy = CheckpointStrategy.Full, fp8: bool = True,
                 fp8_history: int = 16, lr: float = 3e-4, device=None, seed: int = 0,
                 bucket_mb: float = 25.0, loss_scale: Optional[DeviceLossScaleConfig] = None,
                 max_grad_norm: float = 0.0, timed: bool = False, split: str = "balanced",
                 fp8_recipe: str = "tensor", dp_mode: str = "nccl", wire: str = "native", fp8_head: bool = True):
        world = dist.get_world_size()
        if world != dp * pp:
            raise ValueError(f"world size {world} != dp {dp} x pp {pp}")
        if pp > config.num_layers:
            raise ValueError(f"pp {pp} exceeds the layer count {config.num_layers}")
        self.config = config
        self.dp, self.pp = dp, pp
        self.M = num_microbatches
        self.b = micro_batch
        self.S = seq_len or config.max_seq_len
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.layout = PipelineLayout(dp, pp)
        self.rank = dist.get_rank()
        self.replica, self.stage = self.layout.coords(self.rank)
        # every rank creates every group, in the same order
        self.pipe_group = self.grad_group = self.dp_group = None
        for ranks in self.layout.stage_ranks:
            g_act = dist.new_group(ranks)
            g_grad = dist.new_group(ranks)
            if self.rank in ranks:
                self.pipe_group, self.grad_group = g_act, g_grad
        for ranks in self.layout.dp_ranks:
            g = dist.new_group(ranks)
            if self.rank in ranks:
                self.dp_group = g
        if split == "balanced":
            self.split = balanced_split(config, pp, self.S)
        elif split == "even":
            self.split = split_evenly(config.num_layers, pp)
        else:
            raise ValueError(f"unknown split {split!r}")
        lo, hi = self.split[self.stage]
        self.layers = (lo, hi)
        self.is_first, self.is_last = self.stage == 0, self.stage == pp - 1
        torch.manual_seed(seed + self.stage)
        with torch.device(self.device):
            self.model = GptModel(config, init="reference", layers=(lo, hi), embed=self.is_first,
                                  head=self.is_last)
        g = torch.Generator(device=self.device)
        g.manual_seed(seed * 1000 + self.stage)
        self.model.init_normal_(0.02, generator=g)
        if dp_mode not in ("nccl", "symm"):
            raise ValueError(f"dp_mode must be 'nccl' or 'symm', not {dp_mode!r}")
        self.dp_mode = dp_mode if dp > 1 else "none"
        symm = self.dp_mode == "symm"
        self.flat = self.model.flatten(self.device, symmetric=symm, group=self.dp_group if symm else None)
        # the reference GPT's dropout in the kernels; replicas draw different masks, stages
        # differ by their layers' site ids
        self.model.enable_dropout(seed * 1000003 + self.replica)
        self.fp8 = fp8
        if fp8:
            st = self.model.enable_fp8(fp8_history, recipe=fp8_recipe, head=fp8_head)
            if symm:
                from ..ops.fp8 import SymmAmaxSync

                st.set_amax_sync(SymmAmaxSync(self.device, st.cap, self.dp_group))
            elif dp > 1:
                from ..ops.fp8 import NcclAmaxSync

                st.set_amax_sync(NcclAmaxSync(self.dp_group))
        ls = loss_scale or DeviceLossScaleConfig()
        self.reducer = None
        if symm:
            from ..parallel.symm import SymmBucketReducer, ZeroAdam

            self.reducer = SymmBucketReducer(self.flat, self.dp_group, int(bucket_mb * 1024 * 1024))
            self.opt = ZeroAdam(self.flat, self.reducer, lr=lr, max_grad_norm=max_grad_norm, loss_scale=ls)
        else:
            self.opt = FusedAdam(self.flat, lr=lr, max_grad_norm=max_grad_norm, loss_scale=ls)
            if dp > 1:
                from ..parallel.data_parallel import NcclBucketReducer

                self.reducer = NcclBucketReducer(self.flat, self.dp_group, int(bucket_mb * 1024 * 1024))
        b, S = self.b, self.S

        def stage_fn(x):
            return self.model.fused_stage(x, b, S)

        def loss_fn(h, tgt):
            return self.model.fused_head_loss(h, tgt, grad_scale=self.opt.loss_scale_tensor)

        self.executor = DistributedPipelineExecutor(
            self.model, self.layout.stage_ranks[self.replica], schedule, num_microbatches, checkpoint,
            loss_fn=loss_fn, act_shape=(b * S, config.d_model), act_dtype=torch.bfloat16, device=self.device,
            group=self.pipe_group, grad_group=self.grad_group, stage_fn=stage_fn,
            pre_backward=self._pre_backward, sync_losses=False, timed=timed,
            stage_segments=self.model.fused_stage_segments(b, S), wire=wire, pre_forward=self._pre_forward)
        self.schedule = schedule
        self.global_step = 0
        self._loss_host = torch.empty((), dtype=torch.float32).pin_memory()

    def global_name(self, local: str) -> str:
        """Stage parameter name -> the full model's name (``blocks.{j}`` -> ``blocks.{lo+j}``)."""
        if local.startswith("blocks."):
            j, rest = local[len("blocks."):].split(".", 1)
            return f"blocks.{int(j) + self.layers[0]}.{rest}"
        return local

    def state_dict_global(self) -> dict:
        """This stage's parameters under the full model's names (fp32 master copies)."""
        return {self.global_name(k): v.detach() for k, v in self.model.state_dict().items()}

    @torch.no_grad()
    def load_global_state_dict(self, sd: dict) -> None:
        """Load this stage's slice of a full-model state dict (names as in ``GptModel``)."""
        own = self.model.state_dict()
        for k, v in own.items():
            v.copy_(sd[self.global_name(k)].to(v.device, v.dtype))
        self.flat.sync_w16()

    def state_dict(self) -> dict:
        """This rank's stage: weights, Adam state, FP8 state, step (see mtorus.training.checkpoint)."""
        d = {"global_step": self.global_step, "stage": self.stage, "layers": self.layers, "fp8": self.fp8,
             "master": self.flat.master.detach().cpu(), "w16": self.flat.w16.detach().cpu(),
             "opt": {"m": self.opt.m.detach().cpu(), "v": self.opt.v.detach().cpu(),
                     "state": self.opt.state.detach().cpu()}}
        if self.fp8:
            d["fp8_state"] = self.model.fp8_state.state_dict()
        return d

    @torch.no_grad()
    def load_state_dict(self, d: dict) -> None:
        if d["stage"] != self.stage or tuple(d["layers"]) != tuple(self.layers):
            raise ValueError(f"checkpoint holds stage {d['stage']} layers {d['layers']}, "
                             f"this rank runs stage {self.stage} layers {self.layers}")
        self.flat.master.copy_(d["master"].to(self.device))
        self.flat.w16.copy_(d["w16"].to(self.device))
        self.opt.m.copy_(d["opt"]["m"].to(self.device))
        self.opt.v.copy_(d["opt"]["v"].to(self.device))
        self.opt.state.copy_(d["opt"]["state"].to(self.device))
        if self.fp8:
            self.model.fp8_state.load_state_dict(d["fp8_state"])
        self.global_step = int(d["global_step"])

    def ideal_bubble_fraction(self) -> float:
        """(S-1)/(M+S-1) for both schedules (the reference's formula)."""
        return ideal_bubble_fraction(self.pp, self.M)

    def _pre_forward(self, m: int) -> None:
        if self.model.dropout_state is not None:
            self.model.dropout_state.micro = m

    def _pre_backward(self, m: int, k: int) -> None:
        self._pre_forward(m)  # a recomputed forward draws micro-batch m's masks again
        FusedGradState.accumulate = k > 0
        last = k == self.M - 1
        FusedGradState.grad_ready_hook = self.reducer.on_ready if (last and self.reducer is not None) else None

    def step_device(self, ids: Optional[Sequence[torch.Tensor]], targets: Optional[Sequence[torch.Tensor]]):
        """One optimizer step over M micro-batches (device tensors: ``ids`` on the first
        stage, ``targets`` on the last, each a list of M [b, S] tensors).  Returns the
        mean loss as a device scalar on the last stage, None elsewhere; no host sync."""
        loss = self.forward_backward(ids, targets)
        self.optimizer_step()
        return loss

    def warm_kernels(self) -> None:
        """Runs this stage's forward, backward and optimizer kernels once on dummy data,
        with no communication, and restores every piece of state they touch.

        Why: under CUDA lazy module loading (torch's default) the first launch of a
        kernel -- and cuDNN's first use of an attention plan -- may need a context
        synchronisation, which waits for the NCCL receive kernels that this rank
        already has spinning for a neighbour.  If that neighbour is in the same
        situation, both ranks wait forever.  After this call every kernel of the
        step is resident, so the pipelined step never loads code while an NCCL
        kernel is in flight."""
        self._warmed = True
        b, S, d = self.b, self.S, self.config.d_model
        st = self.model.fp8_state if self.fp8 else None
        if st is not None:
            saved = {k: getattr(st, k).clone() for k in ("hist", "amax", "scale", "inv")}
            saved_meta = (st.first_step, set(st._measured), st.cursor)
            self.model.refresh_fp8_weights()
        opt_state = self.opt.state.clone()
        FusedGradState.accumulate = False
        FusedGradState.grad_ready_hook = None
        dev = self.device
        if self.is_first:
            x = torch.zeros((b, S), dtype=torch.long, device=dev)
        else:
            x = torch.zeros((b * S, d), dtype=torch.bfloat16, device=dev, requires_grad=True)
        with torch.no_grad():  # the checkpointed forward
            self.model.fused_stage(x, b, S)
        with torch.enable_grad():
            y = self.model.fused_stage(x, b, S)
            if self.is_last:
                tgt = torch.zeros((b, S), dtype=torch.long, device=dev)
                torch.autograd.backward(self.model.fused_head_loss(y, tgt, grad_scale=self.opt.loss_scale_tensor))
            else:
                torch.autograd.backward(y, torch.zeros_like(y))
        del x, y
        # zero gradients leave master weights and Adam moments unchanged
        self.flat.grad.zero_()
        self.opt.step()
        if st is not None:
            st.end_step()
        with torch.no_grad():
            self.opt.state.copy_(opt_state)
            if st is not None:
                for k, v in saved.items():
                    getattr(st, k).copy_(v)
                st.first_step, st._measured, st.cursor = saved_meta[0], saved_meta[1], saved_meta[2]
        torch.cuda.synchronize(dev)
        # NCCL also connects collective rings / trees on their first use: do that now,
        # at the sizes the step uses, for the data-parallel and the pipeline group
        if self.reducer is not None and self.dp_mode == "nccl":
            s0, e0 = self.reducer.plan.ranges[0]
            tmp = torch.zeros(max(e - s for s, e in self.reducer.plan.ranges), device=dev)
            dist.all_reduce(tmp, group=self.dp_group)
            dist.all_reduce(tmp[:e0 - s0], group=self.dp_group)
            del tmp
        if self.pp > 1:
            dist.all_reduce(torch.zeros(2, device=dev), group=self.pipe_group)
        torch.cuda.synchronize(dev)

    def forward_backward(self, ids, targets):
        """The schedule's forwards / backwards and the data-parallel reduction: leaves
        the step's averaged gradients in ``flat.grad``; returns the device loss (last
        stage) or None."""
        if not getattr(self, "_warmed", False):
            self.warm_kernels()
        if self.fp8:
            self.model.refresh_fp8_weights()
        if hasattr(self.reducer, "begin_step"):
            self.reducer.begin_step()
        loss = self.executor.run(ids if self.is_first else None, targets if self.is_last else None)
        FusedGradState.grad_ready_hook = None
        FusedGradState.accumulate = False
        if self.reducer is not None:
            self.reducer.finish()
        return loss

    def optimizer_step(self) -> None:
        """Pipeline-wide norm / overflow, then the fused Adam update and the FP8 scale roll."""
        if self.dp_mode != "symm":  # the symmetric reduce kernels already summed this stage's norm partials
            self.opt.accumulate_norm()
        if self.pp > 1:
            # sum of squares and the non-finite count over the whole model
            dist.all_reduce(self.opt.state[ST_SUMSQ:ST_NONFINITE + 1], group=self.pipe_group)
        self.opt.finalize()
        self.opt.update()
        if self.fp8:
            self.model.fp8_state.end_step()
        if self.model.dropout_state is not None:
            self.model.dropout_state.micro = 0
            self.model.dropout_state.advance()
        self.global_step += 1

    def train_step(self, ids_host: Optional[torch.Tensor], targets_host: Optional[torch.Tensor]) -> Optional[float]:
        """Host batch [M, b, S] in (pinned; ids needed on the first stage, targets on the
        last), host mean loss out on the last stage (None elsewhere)."""
        ids = tgt = None
        if self.is_first:
            d = ids_host.to(self.device, non_blocking=True)
            ids = list(d.unbind(0))
        if self.is_last:
            d = targets_host.to(self.device, non_blocking=True)
            tgt = list(d.unbind(0))
        loss = self.step_device(ids, tgt)
        if loss is None:
            return None
        self._loss_host.copy_(loss, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return float(self._loss_host)


__all__ = ["PipelineLayout", "PipelineTrainer", "balanced_split", "stage_costs"]
