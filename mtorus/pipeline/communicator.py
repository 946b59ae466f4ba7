"""FP8-compressed stage-to-stage transfer.

Reference: crates/mt-pipeline/src/communicator.rs.  Activations and gradients
are quantised per tensor (the reference uses the same format, E4M3 by default,
for both) and framed as ``rows u64 | cols u64 | format u8 | scale f32 | len u64
| fp8 bytes`` (29-byte header); the codec and framing are C++.
"""
from __future__ import annotations

from .._ext import host as _host
from .stage import StageData

_C = _host()


class PipelineComm:
    def __init__(self, comm, fp8_format=None):
        self.comm = comm
        self.fp8_format = fp8_format if fp8_format is not None else _C.Fp8Format.E4M3

    def with_fp8_format(self, fmt) -> "PipelineComm":
        self.fp8_format = fmt
        return self

    def compress_stage_data(self, data: StageData) -> bytes:
        return _C.compress_stage_data(data.values, data.rows, data.cols, self.fp8_format)

    @staticmethod
    def decompress_stage_data(b: bytes) -> StageData:
        v, r, c = _C.decompress_stage_data(b)
        return StageData(v, r, c)

    def send_activations(self, data: StageData, dst_stage: int) -> None:
        self.comm.send(self.compress_stage_data(data), dst_stage)

    def recv_activations(self, src_stage: int) -> StageData:
        return self.decompress_stage_data(self.comm.recv(src_stage))

    def send_gradients(self, data: StageData, dst_stage: int) -> None:
        self.comm.send(self.compress_stage_data(data), dst_stage)

    def recv_gradients(self, src_stage: int) -> StageData:
        return self.decompress_stage_data(self.comm.recv(src_stage))

    def rank(self) -> int:
        return self.comm.rank()

    def world_size(self) -> int:
        return self.comm.world_size()


__all__ = ["PipelineComm"]
