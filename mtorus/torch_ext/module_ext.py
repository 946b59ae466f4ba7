"""Splitting torch modules into pipeline stages.

Reference: crates/mt-burn/src/module_ext.rs -- ``StageForward`` (forward only),
named ``PipelineStage``, the ``PipelineModule::split_into_stages`` trait (no
implementors in the reference; implemented here for ``nn.Sequential`` and the
GPT model), ``SequentialStages`` and ``split_evenly`` (the first count % S
stages get one extra layer; S is clamped to count; zero -> empty).
"""
from __future__ import annotations

import abc
from typing import List, Optional, Sequence, Tuple

import torch


def split_evenly(count: int, num_stages: int) -> List[Tuple[int, int]]:
    if num_stages == 0 or count == 0:
        return []
    n = min(num_stages, count)
    base, rem = divmod(count, n)
    out, off = [], 0
    for i in range(n):
        ln = base + (1 if i < rem else 0)
        out.append((off, off + ln))
        off += ln
    return out


class StageForward(abc.ABC):
    @abc.abstractmethod
    def forward(self, x: torch.Tensor) -> torch.Tensor: ...


class ModuleStage(StageForward):
    def __init__(self, module: torch.nn.Module):
        self.module = module

    def forward(self, x):
        return self.module(x)


class PipelineStage:
    def __init__(self, name: str, inner):
        self._name = name
        self.inner = inner

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.inner.forward(x) if hasattr(self.inner, "forward") else self.inner(x)

    def __call__(self, x):
        return self.forward(x)

    def name(self) -> str:
        return self._name


class PipelineModule(abc.ABC):
    @abc.abstractmethod
    def split_into_stages(self, num_stages: int) -> List[PipelineStage]: ...


class SequentialStages:
    def __init__(self, stages: Sequence[PipelineStage]):
        self.stages = list(stages)

    def forward(self, x):
        for s in self.stages:
            x = s.forward(x)
        return x

    def stage(self, i: int) -> Optional[PipelineStage]:
        return self.stages[i] if 0 <= i < len(self.stages) else None

    def num_stages(self) -> int:
        return len(self.stages)


def split_sequential(seq: torch.nn.Sequential, num_stages: int) -> List[PipelineStage]:
    layers = list(seq.children())
    return [PipelineStage(f"stage_{i}", ModuleStage(torch.nn.Sequential(*layers[a:b])))
            for i, (a, b) in enumerate(split_evenly(len(layers), num_stages))]


__all__ = ["split_evenly", "StageForward", "ModuleStage", "PipelineStage", "PipelineModule", "SequentialStages",
           "split_sequential"]
