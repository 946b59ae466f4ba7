"""Gradient accumulation across micro-batches.

Reference: crates/mt-training/src/accumulator.rs.  Gradients are summed per
parameter id in fp32.  Counting semantics are kept: ``register`` /
``register_values`` add 1 per call (per parameter), ``drain_from`` adds 1 per
call (per micro-batch) and returns the L2 norm of what it drained.  The sums
stay on the device of the incoming tensors (the reference copies every gradient
to host memory).

The fused GPT path does not use this class: its GEMM epilogues accumulate
straight into the flat fp32 gradient buffer.
"""
from __future__ import annotations

import itertools
from typing import Dict, Iterable, List, Optional

import torch

_ids = itertools.count(1)


class ParamId:
    __slots__ = ("value",)

    def __init__(self, value: int):
        self.value = int(value)

    def __hash__(self):
        return hash(self.value)

    def __eq__(self, o):
        return isinstance(o, ParamId) and o.value == self.value

    def __repr__(self):
        return f"ParamId({self.value})"


def param_id(p: torch.nn.Parameter) -> ParamId:
    pid = getattr(p, "_mt_param_id", None)
    if pid is None:
        pid = ParamId(next(_ids))
        p._mt_param_id = pid
    return pid


def list_param_ids(module: torch.nn.Module) -> List[ParamId]:
    return [param_id(p) for p in module.parameters()]


class GradientsParams(dict):
    """Parameter id -> gradient tensor (burn-optim's GradientsParams)."""

    def register(self, pid: ParamId, t: torch.Tensor) -> None:
        self[pid] = t

    def remove(self, pid: ParamId) -> Optional[torch.Tensor]:
        return self.pop(pid, None)

    @staticmethod
    def from_module(module: torch.nn.Module) -> "GradientsParams":
        gp = GradientsParams()
        for p in module.parameters():
            if p.grad is not None:
                gp.register(param_id(p), p.grad.detach().reshape(-1))
        return gp


class GradientAccumulator:
    def __init__(self, device=None):
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self._grads: Dict[ParamId, torch.Tensor] = {}
        self.count = 0

    def _store(self, pid: ParamId, values: torch.Tensor) -> None:
        v = values.detach().reshape(-1).to(torch.float32)
        cur = self._grads.get(pid)
        if cur is None:
            self._grads[pid] = v.clone()
        else:
            if cur.numel() != v.numel():
                raise ValueError(f"gradient size mismatch for param {pid}")
            cur.add_(v.to(cur.device))
        self.count += 1

    def register(self, pid: ParamId, grad: torch.Tensor) -> float:
        """Adds grad; returns its squared L2 norm.  count += 1."""
        g = torch.as_tensor(grad)
        self._store(pid, g)
        return float(g.float().pow(2).sum())

    def register_values(self, pid: ParamId, values) -> None:
        self._store(pid, torch.as_tensor(values, dtype=torch.float32))

    def drain_from(self, grads: GradientsParams, param_ids: Iterable[ParamId]) -> float:
        """Moves every listed gradient out of ``grads`` into the sums; count += 1;
        returns the L2 norm of the drained gradients."""
        sq = None
        for pid in param_ids:
            t = grads.remove(pid)
            if t is None:
                continue
            v = t.detach().reshape(-1).to(torch.float32)
            s = v.pow(2).sum()
            sq = s if sq is None else sq + s.to(sq.device)
            cur = self._grads.get(pid)
            if cur is None:
                self._grads[pid] = v.clone()
            else:
                cur.add_(v.to(cur.device))
        self.count += 1
        return 0.0 if sq is None else float(sq.sqrt())

    def reset(self) -> None:
        self._grads.clear()
        self.count = 0

    def step_count(self) -> int:
        return self.count

    def effective_batch_size(self, micro_batch_size: int) -> int:
        return micro_batch_size * self.count

    def into_gradients(self) -> GradientsParams:
        gp = GradientsParams()
        for pid, v in self._grads.items():
            gp.register(pid, v)
        self._grads = {}
        return gp

    def raw_grads(self) -> Dict[ParamId, torch.Tensor]:
        return self._grads

    def raw_grads_mut(self) -> Dict[ParamId, torch.Tensor]:
        return self._grads

    def __repr__(self) -> str:
        return f"GradientAccumulator {{ param_count: {len(self._grads)}, count: {self.count} }}"


__all__ = ["ParamId", "param_id", "list_param_ids", "GradientsParams", "GradientAccumulator"]
