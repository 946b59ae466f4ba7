"""GptTrainer: the end-to-end public training API of the fused B200 path.

    trainer = GptTrainer(GptConfig.gpt_1b_bench(), device="cuda:0")
    loss = trainer.train_step(input_ids_cpu, targets_cpu)   # host tensors in, float out

One step = H2D copy of the batch (pinned, non-blocking) -> fused forward/backward
(gradients land in the flat fp32 buffer) -> data-parallel bucket reduction
overlapped with backward (when a process group is given) -> device-resident
optimizer (norm, overflow, loss scale, clip, Adam) -> D2H read of the loss.

This is the executable form of the reference's training path
(examples/gpt-1b/src/main.rs:96-115 and crates/mt-training/src/step.rs:114-180),
with the gradient all-reduce the reference leaves out.
"""
from __future__ import annotations

from typing import Optional

import torch

from ..models.gpt import GptConfig, GptModel
from ..ops.fused import FusedGradState
from .fused_optim import DeviceLossScaleConfig, FusedAdam


class GptTrainer:
    def __init__(self, config: GptConfig, device="cuda", lr: float = 3e-4, init: str = "normal",
                 seed: int = 0, dp_group=None, dp: str = "nccl", bucket_mb: float = 25.0,
                 loss_scale: Optional[DeviceLossScaleConfig] = None, max_grad_norm: float = 0.0,
                 weight_decay: float = 0.0, warmup_steps: int = 0, fp8: bool = False,
                 fp8_history: int = 16, fp8_recipe: str = "tensor", fp8_head: bool = True):
        self.config = config
        self.device = torch.device(device)
        torch.manual_seed(seed)
        with torch.device(self.device):
            self.model = GptModel(config, init="reference")
        if init == "normal":
            g = torch.Generator(device=self.device)
            g.manual_seed(seed)
            self.model.init_normal_(0.02, generator=g)
        multi = dp_group is not None or (torch.distributed.is_initialized() and torch.distributed.get_world_size() > 1)
        self.dp = dp if multi else "none"
        self.flat = self.model.flatten(self.device, symmetric=self.dp == "symm", group=dp_group)
        # the reference GPT's dropout (p = config.dropout at its five sites), drawn in the kernels;
        # ranks draw different masks (the seed folds in the data-parallel rank)
        dp_rank = torch.distributed.get_rank(dp_group) if multi else 0
        self.model.enable_dropout(seed * 1000003 + dp_rank)
        self.lr = lr
        self.warmup_steps = warmup_steps
        self.global_step = 0
        self.reducer = None
        ls = loss_scale or DeviceLossScaleConfig()
        self.fp8 = fp8
        if fp8:
            st = self.model.enable_fp8(fp8_history, recipe=fp8_recipe, head=fp8_head)
            if self.dp == "symm":
                from ..ops.fp8 import SymmAmaxSync

                st.set_amax_sync(SymmAmaxSync(self.device, st.cap, dp_group))
            elif self.dp == "nccl":
                from ..ops.fp8 import NcclAmaxSync

                st.set_amax_sync(NcclAmaxSync(dp_group))
        if self.dp == "symm":
            from ..parallel.symm import SymmBucketReducer, ZeroAdam

            self.reducer = SymmBucketReducer(self.flat, dp_group, int(bucket_mb * 1024 * 1024))
            self.opt = ZeroAdam(self.flat, self.reducer, lr=lr, max_grad_norm=max_grad_norm,
                                weight_decay=weight_decay, loss_scale=ls)
        else:
            self.opt = FusedAdam(self.flat, lr=lr, max_grad_norm=max_grad_norm, weight_decay=weight_decay,
                                 loss_scale=ls)
            if self.dp == "nccl":
                from ..parallel.data_parallel import NcclBucketReducer

                self.reducer = NcclBucketReducer(self.flat, dp_group, int(bucket_mb * 1024 * 1024))
            elif self.dp != "none":
                raise ValueError(f"unknown dp reducer {dp!r}")
        self._ids = None
        self._tgt = None
        self._loss_host = torch.empty((), dtype=torch.float32).pin_memory() if torch.cuda.is_available() else None

    def current_lr(self) -> float:
        """Linear warmup (reference step.rs:146-150), then constant."""
        if self.warmup_steps > 0 and self.global_step < self.warmup_steps:
            return self.lr * (self.global_step + 1) / self.warmup_steps
        return self.lr

    def step_device_accum(self, ids_list, targets_list) -> torch.Tensor:
        """One optimizer step over several micro-batches (gradient accumulation:
        the reference's GradientAccumulator, crates/mt-training/src/accumulator.rs).
        The first micro-batch's backward overwrites ``main_grad``, the others add
        into it in the wgrad epilogues; the data-parallel reduction runs during the
        last backward.  Returns the mean loss as a device scalar."""
        k = len(ids_list)
        if k == 1:
            return self.step_device(ids_list[0], targets_list[0])
        if self.fp8:
            self.model.refresh_fp8_weights()
        if hasattr(self.reducer, "begin_step"):
            self.reducer.begin_step()
        gs = self.opt.loss_scale_tensor / k
        total = None
        ds = self.model.dropout_state
        for i, (ids, tgt) in enumerate(zip(ids_list, targets_list)):
            if ds is not None:
                ds.micro = i
            FusedGradState.accumulate = i > 0
            last = i == k - 1
            FusedGradState.grad_ready_hook = self.reducer.on_ready if (last and self.reducer is not None) else None
            loss = self.model.fused_loss(ids, tgt, grad_scale=gs)
            loss.backward()
            total = loss.detach() if total is None else total + loss.detach()
        FusedGradState.accumulate = False
        FusedGradState.grad_ready_hook = None
        if self.reducer is not None:
            self.reducer.finish()
        self.opt.step(self.current_lr())
        if self.fp8:
            self.model.fp8_state.end_step()
        if ds is not None:
            ds.micro = 0
            ds.advance()
        self.global_step += 1
        return total / k

    def step_device(self, ids: torch.Tensor, targets: torch.Tensor, reduce: bool = True) -> torch.Tensor:
        """One full training step on device tensors; returns the device loss (no sync).

        ``reduce=False`` runs the same step with no data-parallel communication at
        all (each rank updates its own replica with a local Adam): the compute-only
        reference against which the exposed communication time of a real step is
        measured.  Every rank must pass the same value."""
        FusedGradState.accumulate = False
        if self.fp8:
            self.model.refresh_fp8_weights()
        reducer = self.reducer if reduce else None
        FusedGradState.grad_ready_hook = reducer.on_ready if reducer is not None else None
        if hasattr(reducer, "begin_step"):
            reducer.begin_step()
        opt = self.opt if reduce or self.reducer is None else self._local_optimizer()
        loss = self.model.fused_loss(ids, targets, grad_scale=opt.loss_scale_tensor)
        loss.backward()
        if reducer is not None:
            reducer.finish()
        FusedGradState.grad_ready_hook = None
        opt.step(self.current_lr())
        if self.fp8:
            self.model.fp8_state.end_step()
        if self.model.dropout_state is not None:
            self.model.dropout_state.advance()  # next step's masks (on the device: graph-safe)
        self.global_step += 1
        return loss.detach()

    # ---------------------------------------------------------------- checkpoints
    def state_dict(self) -> dict:
        """Everything this rank needs to resume bit for bit (see mtorus.training.checkpoint)."""
        opt = self.opt
        d = {"global_step": self.global_step, "dp": self.dp, "fp8": self.fp8,
             "master": self.flat.master.detach().cpu(), "w16": self.flat.w16.detach().cpu(),
             "opt": {"m": opt.m.detach().cpu(), "v": opt.v.detach().cpu(), "state": opt.state.detach().cpu()}}
        if self.fp8:
            d["fp8_state"] = self.model.fp8_state.state_dict()
        if self.model.dropout_state is not None:
            d["dropout_rng"] = self.model.dropout_state.rng.detach().cpu()
        return d

    @torch.no_grad()
    def load_state_dict(self, d: dict) -> None:
        if d["dp"] != self.dp or bool(d["fp8"]) != bool(self.fp8):
            raise ValueError(f"checkpoint was written with dp={d['dp']} fp8={d['fp8']}, "
                             f"this trainer has dp={self.dp} fp8={self.fp8}")
        self.flat.master.copy_(d["master"].to(self.device))
        self.flat.w16.copy_(d["w16"].to(self.device))
        self.opt.m.copy_(d["opt"]["m"].to(self.device))
        self.opt.v.copy_(d["opt"]["v"].to(self.device))
        self.opt.state.copy_(d["opt"]["state"].to(self.device))
        if self.fp8:
            self.model.fp8_state.load_state_dict(d["fp8_state"])
        if self.model.dropout_state is not None and "dropout_rng" in d:
            ds = self.model.dropout_state
            ds.rng.copy_(d["dropout_rng"].to(ds.rng.device))
            ds.step = (int(d["dropout_rng"][2]) & 0xFFFFFFFF) | ((int(d["dropout_rng"][3]) & 0xFFFFFFFF) << 32)
        self.global_step = int(d["global_step"])

    def _local_optimizer(self) -> FusedAdam:
        if getattr(self, "_local_opt", None) is None:
            self._local_opt = FusedAdam(self.flat, lr=self.lr)
        return self._local_opt

    # ---------------------------------------------------------------- CUDA graph
    def capture(self, ids: torch.Tensor, targets: torch.Tensor, reduce: bool = True) -> int:
        """Captures one whole training step (forward, backward, data-parallel bucket
        all-reduce, optimizer, FP8 scale roll) into a CUDA graph over static input
        buffers shaped like ``ids`` / ``targets``; ``graph_step`` then replays it with
        one launch instead of ~1000.  Call after at least one eager step (the FP8
        first-step path and every kernel's one-time set-up must have run).  Any
        data-parallel mode: NCCL buckets, or the symmetric-memory path, whose flag
        epochs and amax stamps come from device step counters that the captured
        step advances itself.  Returns the number of this framework's kernels in
        the graph."""
        from .._ext import cuda as _cuda

        if self.global_step == 0 or (self.fp8 and self.model.fp8_state.first_step):
            raise RuntimeError("run one eager step before capturing")
        if self.warmup_steps and self.global_step < self.warmup_steps:
            raise RuntimeError("the learning rate is still warming up (it is baked into the graph)")
        if not reduce:
            self._local_optimizer()  # its state must exist outside the graph
        if getattr(self, "_g_ids", None) is None or self._g_ids.shape != ids.shape:
            self._g_ids = ids.detach().clone()
            self._g_tgt = targets.detach().clone()
        torch.cuda.synchronize()
        lc0 = _cuda().launch_count()
        g = torch.cuda.CUDAGraph()
        step0 = self.global_step
        cursor0 = self.model.fp8_state.cursor if self.fp8 else None
        with torch.cuda.graph(g):
            loss = self.step_device(self._g_ids, self._g_tgt, reduce=reduce)
        self.global_step = step0  # capture records, it does not run a step
        if self.fp8:
            self.model.fp8_state.cursor = cursor0
        if self.model.dropout_state is not None:
            self.model.dropout_state.step -= 1
        n = int(_cuda().launch_count() - lc0)
        if not hasattr(self, "_graphs"):
            self._graphs = {}
        self._graphs[reduce] = (g, loss, n)
        if reduce:
            self._graph, self._g_loss, self.graph_launches = g, loss, n
        torch.cuda.synchronize()
        return n

    def release_graphs(self) -> None:
        """Drop the captured step graphs (call before destroying a process group
        whose NCCL calls a graph holds)."""
        torch.cuda.synchronize()
        self._graphs = {}
        self._graph = self._g_loss = None

    def graph_step(self, ids: torch.Tensor, targets: torch.Tensor, reduce: bool = True) -> torch.Tensor:
        """One training step by replaying the captured graph; returns the device loss."""
        g, loss, _ = self._graphs[reduce]
        self._g_ids.copy_(ids, non_blocking=True)
        self._g_tgt.copy_(targets, non_blocking=True)
        g.replay()
        self.global_step += 1
        if self.fp8:
            st = self.model.fp8_state
            st.cursor = (st.cursor + 1) % st.history
        if self.model.dropout_state is not None:
            self.model.dropout_state.step += 1
        return loss

    def train_step(self, input_ids: torch.Tensor, targets: torch.Tensor) -> float:
        """Host batch in (ideally pinned), host loss out."""
        if self._ids is None or self._ids.shape != input_ids.shape:
            self._ids = torch.empty(input_ids.shape, dtype=torch.long, device=self.device)
            self._tgt = torch.empty(targets.shape, dtype=torch.long, device=self.device)
        if getattr(self, "_graph", None) is not None and input_ids.shape == self._g_ids.shape:
            loss = self.graph_step(input_ids, targets)  # host -> static buffers, replay
        else:
            self._ids.copy_(input_ids, non_blocking=True)
            self._tgt.copy_(targets, non_blocking=True)
            loss = self.step_device(self._ids, self._tgt)
        self._loss_host.copy_(loss, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return float(self._loss_host)
