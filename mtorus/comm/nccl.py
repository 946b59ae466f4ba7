"""Communicator over torch.distributed process groups (NCCL on GPUs, gloo on CPU).

Implements the byte-level ``Communicator`` interface (so it plugs into
``TopologyAwareComm``, ``PipelineComm`` and ``DistributedRuntime``) and the
tensor-level collectives the training path uses.  With the NCCL backend this is
the library baseline; the fused NVLink kernels are in ``mtorus.parallel.symm``.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from .base import Communicator, DType, ReduceOp

_TORCH_DT = {DType.U64: torch.int64, DType.I64: torch.int64, DType.F32: torch.float32, DType.F64: torch.float64,
             DType.I32: torch.int32, DType.U8: torch.uint8}
_OPS = {ReduceOp.Sum: dist.ReduceOp.SUM, ReduceOp.Product: dist.ReduceOp.PRODUCT, ReduceOp.Min: dist.ReduceOp.MIN,
        ReduceOp.Max: dist.ReduceOp.MAX, ReduceOp.Mean: dist.ReduceOp.SUM}


class DistCommunicator(Communicator):
    def __init__(self, group=None, device: Optional[torch.device] = None):
        Communicator.__init__(self)
        self.group = group
        self._rank = dist.get_rank(group)
        self._world = dist.get_world_size(group)
        self._backend = dist.get_backend(group)
        if device is None:
            device = (torch.device("cuda", torch.cuda.current_device()) if self._backend == "nccl"
                      else torch.device("cpu"))
        self.device = device
        self._pending = []

    # ------------------------------------------------------------ helpers
    def _g(self, r: int) -> int:
        return r if self.group is None else dist.get_global_rank(self.group, r)

    def _to_tensor(self, data: bytes) -> torch.Tensor:
        t = torch.frombuffer(bytearray(data), dtype=torch.uint8) if data else torch.empty(0, dtype=torch.uint8)
        return t.to(self.device)

    # ------------------------------------------------------------ Communicator
    def send(self, data: bytes, dst: int) -> None:
        # Posted asynchronously (the Communicator contract lets every rank send
        # before it receives); buffers stay referenced until the transfer ends.
        n = torch.tensor([len(data)], dtype=torch.int64, device=self.device)
        self._pending.append((dist.isend(n, self._g(dst), group=self.group), n))
        if data:
            t = self._to_tensor(data)
            self._pending.append((dist.isend(t, self._g(dst), group=self.group), t))
        self._pending = [(w, t) for w, t in self._pending if not w.is_completed()]

    def flush(self) -> None:
        for w, _ in self._pending:
            w.wait()
        self._pending = []

    def recv(self, src: int) -> bytes:
        n = torch.empty(1, dtype=torch.int64, device=self.device)
        dist.recv(n, self._g(src), group=self.group)
        k = int(n.item())
        if k == 0:
            return b""
        buf = torch.empty(k, dtype=torch.uint8, device=self.device)
        dist.recv(buf, self._g(src), group=self.group)
        return bytes(buf.cpu().numpy().tobytes())

    def all_reduce(self, data: bytes, op=ReduceOp.Sum, dtype=DType.U64) -> bytes:
        tdt = _TORCH_DT[dtype]
        es = torch.empty(0, dtype=tdt).element_size()
        n = len(data) // es
        t = torch.frombuffer(bytearray(data[:n * es]), dtype=tdt).clone().to(self.device) if n else \
            torch.empty(0, dtype=tdt, device=self.device)
        dist.all_reduce(t, op=_OPS[op], group=self.group)
        if op == ReduceOp.Mean:
            t = t.div(self._world, rounding_mode="floor") if not t.is_floating_point() else t / self._world
        return bytes(t.cpu().numpy().tobytes())

    def broadcast(self, data: bytes, root: int) -> bytes:
        n = torch.tensor([len(data)], dtype=torch.int64, device=self.device)
        dist.broadcast(n, self._g(root), group=self.group)
        k = int(n.item())
        buf = self._to_tensor(data) if self._rank == root else torch.empty(k, dtype=torch.uint8, device=self.device)
        if k:
            dist.broadcast(buf, self._g(root), group=self.group)
        return bytes(buf.cpu().numpy().tobytes())

    def all_gather(self, data: bytes) -> List[bytes]:
        n = torch.tensor([len(data)], dtype=torch.int64, device=self.device)
        ns = [torch.empty_like(n) for _ in range(self._world)]
        dist.all_gather(ns, n, group=self.group)
        sizes = [int(x.item()) for x in ns]
        mx = max(sizes) if sizes else 0
        buf = torch.zeros(mx, dtype=torch.uint8, device=self.device)
        if data:
            buf[:len(data)] = self._to_tensor(data)
        outs = [torch.empty_like(buf) for _ in range(self._world)]
        if mx:
            dist.all_gather(outs, buf, group=self.group)
        return [bytes(o[:s].cpu().numpy().tobytes()) for o, s in zip(outs, sizes)]

    def barrier(self) -> None:
        self.flush()
        dist.barrier(group=self.group)

    def rank(self) -> int:
        return self._rank

    def world_size(self) -> int:
        return self._world

    def backend(self) -> str:
        return self._backend

    # ------------------------------------------------------------ tensor API
    def all_reduce_tensor(self, t: torch.Tensor, op=dist.ReduceOp.SUM, async_op: bool = False):
        return dist.all_reduce(t, op=op, group=self.group, async_op=async_op)

    def reduce_scatter_tensor(self, out: torch.Tensor, inp: torch.Tensor, op=dist.ReduceOp.SUM, async_op=False):
        return dist.reduce_scatter_tensor(out, inp, op=op, group=self.group, async_op=async_op)

    def all_gather_tensor(self, out: torch.Tensor, inp: torch.Tensor, async_op: bool = False):
        return dist.all_gather_into_tensor(out, inp, group=self.group, async_op=async_op)

    def broadcast_tensor(self, t: torch.Tensor, root: int, async_op: bool = False):
        return dist.broadcast(t, self._g(root), group=self.group, async_op=async_op)

    def send_tensor(self, t: torch.Tensor, dst: int):
        return dist.isend(t, self._g(dst), group=self.group)

    def recv_tensor(self, t: torch.Tensor, src: int):
        return dist.irecv(t, self._g(src), group=self.group)


NcclCommunicator = DistCommunicator

__all__ = ["DistCommunicator", "NcclCommunicator"]
