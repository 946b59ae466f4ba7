"""Pipeline stages over fp32 row-major blobs (the reference's simulation types).

Reference: crates/mt-pipeline/src/stage.rs.  ``StageData`` is an fp32 matrix
with the wire format ``rows u64 | cols u64 | f32 values`` (little endian).
``PipelineStage.backward`` hands the *stage input* to every layer in reverse
order, as the reference does (stage.rs:100-106).

The multi-GPU executor (``mtorus.pipeline.executor.DistributedPipelineExecutor``)
works on torch modules and tensors instead; these types back the reference's
single-process simulated executor and its tests.
"""
from __future__ import annotations

import abc
from typing import Callable, List, Optional, Sequence

from .._ext import host as _host

_C = _host()


class StageData:
    __slots__ = ("values", "rows", "cols")

    def __init__(self, values: Sequence[float], rows: int, cols: int):
        values = [float(v) for v in values]
        if len(values) != rows * cols:
            raise ValueError("data length mismatch")
        self.values = values
        self.rows = rows
        self.cols = cols

    @staticmethod
    def zeros(rows: int, cols: int) -> "StageData":
        return StageData([0.0] * (rows * cols), rows, cols)

    def __len__(self) -> int:
        return len(self.values)

    def len(self) -> int:
        return len(self.values)

    def is_empty(self) -> bool:
        return not self.values

    def to_bytes(self) -> bytes:
        return _C.stage_data_to_bytes(self.values, self.rows, self.cols)

    @staticmethod
    def from_bytes(b: bytes) -> "StageData":
        v, r, c = _C.stage_data_from_bytes(b)
        return StageData(v, r, c)

    def clone(self) -> "StageData":
        return StageData(list(self.values), self.rows, self.cols)

    def __eq__(self, o) -> bool:
        return isinstance(o, StageData) and (self.values, self.rows, self.cols) == (o.values, o.rows, o.cols)

    def __repr__(self) -> str:
        return f"StageData(rows={self.rows}, cols={self.cols})"


class StageForward(abc.ABC):
    @abc.abstractmethod
    def forward(self, input: StageData) -> StageData: ...

    @abc.abstractmethod
    def backward(self, input: StageData, grad_output: StageData) -> StageData: ...


class StageForwardClosure(StageForward):
    def __init__(self, forward_fn: Callable, backward_fn: Callable):
        self.forward_fn = forward_fn
        self.backward_fn = backward_fn

    def forward(self, input: StageData) -> StageData:
        return self.forward_fn(input)

    def backward(self, input: StageData, grad_output: StageData) -> StageData:
        return self.backward_fn(input, grad_output)


class PipelineStage:
    def __init__(self, stage_id: int, layers: List[StageForward]):
        self.stage_id = stage_id
        self.layers = list(layers)
        self.input_cache: Optional[StageData] = None
        self.activation_buffer: List[StageData] = []

    def forward(self, input: StageData) -> StageData:
        out = input
        for layer in self.layers:
            out = layer.forward(out)
        return out

    def backward(self, input: StageData, grad_output: StageData) -> StageData:
        grad = grad_output
        for layer in reversed(self.layers):
            grad = layer.backward(input.clone(), grad)
        return grad

    def checkpoint_forward(self, input: StageData) -> StageData:
        self.input_cache = input.clone()
        return self.forward(input)

    def recompute_and_backward(self, grad_output: StageData) -> StageData:
        if self.input_cache is None:
            raise RuntimeError("no cached input for recomputation")
        inp, self.input_cache = self.input_cache, None
        self.forward(inp.clone())
        return self.backward(inp, grad_output)

    def num_layers(self) -> int:
        return len(self.layers)


__all__ = ["StageData", "StageForward", "StageForwardClosure", "PipelineStage"]
