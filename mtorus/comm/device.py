"""Device communicator: the ``Communicator`` interface over NVLink peer memory.

``SymmCommunicator`` implements the reference's communicator surface
(crates/mt-comm/src/collective.rs:3-32: send / recv / all_reduce / broadcast /
all_gather / rank / world_size, ReduceOp Sum / Product / Min / Max / Mean) with
this framework's own kernels on symmetric (peer-mapped) memory, one process per
GPU, no NCCL on the data path:

* every collective stages this rank's message in a symmetric byte buffer
  (``[int64 length | 8 pad | payload]``), meets the other ranks at a flag
  barrier, and pulls the messages it needs straight from the peers' staging
  buffers over NVLink (``symm_pull_msgs``); ``all_reduce`` reads every peer's
  message and reduces it element by element in rank order
  (``symm_allreduce_msgs``), the order of the host ``reduce_buffers``, so float
  sums agree bit for bit with the CPU communicators;
* ``exchange`` (used by ``TopologyAwareComm.exchange_with_neighbors`` and
  ``nearest_neighbor_exchange``) pulls one message from each torus neighbour in a
  single kernel (reference crates/mt-comm/src/topology_aware.rs:38-49);
* ``send`` / ``recv`` go through a mailbox ring in the receiver's symmetric
  memory: the sender copies the message into the ring slot (copy engine, over
  NVLink) and release-stores a sequence number into the receiver's flag; the
  receiver waits for it, reads the slot and acknowledges; at most ``ring``
  messages per ordered pair are in flight, in order.

Every device wait is bounded (5 s); a wait that runs out records a status code
and the host call raises ``CommTimeout``.  Collectives (all_reduce, broadcast,
all_gather, exchange, barrier) must be called by every rank of the group in the
same order.

The tensor methods (``all_reduce_tensor``, ``all_gather_tensor``,
``broadcast_tensor``, ``exchange_neighbors_tensor``) keep the data on the device
and use the bandwidth kernels of ``mtorus.parallel.symm.SymmCollectives``
(NVLS ``multimem`` reduction when the fabric offers it, else two-shot peer
loads; the torus halo as direct peer stores).
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from .._ext import cuda as _cuda
from .base import CommError, CommTimeout, Communicator, DType, ReduceOp

_HDR = 16
_DT_CODE = {DType.U64: 0, DType.I64: 1, DType.F32: 2, DType.F64: 3, DType.I32: 4, DType.U8: 5}
_OP_CODE = {ReduceOp.Sum: 0, ReduceOp.Product: 1, ReduceOp.Min: 2, ReduceOp.Max: 3, ReduceOp.Mean: 4}


def _round16(n: int) -> int:
    return (n + 15) // 16 * 16


class SymmCommunicator(Communicator):
    """Communicator of one process per GPU over symmetric memory (see module doc).

    group      torch.distributed process group whose ranks share the NVLink fabric
               (default: the world); its store exchanges the peer mappings once
    max_bytes  largest message of the byte interface
    ring       point-to-point messages in flight per ordered pair of ranks
    tensor_bytes  capacity of the tensor collectives' buffers (0: no tensor API)
    """

    def __init__(self, group=None, device=None, max_bytes: int = 16 << 20, ring: int = 4,
                 tensor_bytes: int = 64 << 20, ctas: int = 32):
        Communicator.__init__(self)
        from ..parallel.symm import SymmBuffer, SymmContext

        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.group = group
        self.cap = _round16(max_bytes)
        self.slot = self.cap + _HDR
        self.ring = ring
        self.ctas = ctas
        self.ctx = SymmContext(self.device, group, num_slots=8)
        self._rank, self._world = self.ctx.rank, self.ctx.world
        n = self._world
        self.stage = SymmBuffer(self.slot, torch.uint8, self.device, group, zero=True)
        self.mail = SymmBuffer(n * ring * self.slot, torch.uint8, self.device, group, zero=True)
        self.pflags = SymmBuffer(2 * n, torch.int32, self.device, group, zero=True)
        self.sendbuf = torch.zeros(self.slot, dtype=torch.uint8, device=self.device)
        self.inbox = torch.zeros(max(n, 16) * self.slot, dtype=torch.uint8, device=self.device)
        self.epoch = 0
        self.sent = [0] * n
        self.recvd = [0] * n
        self.coll = None
        if tensor_bytes:
            from ..parallel.symm import SymmCollectives

            self.coll = SymmCollectives(self.device, group, max_bytes=_round16(tensor_bytes), ctas=128)
        self.ctx.flags.barrier()

    # ------------------------------------------------------------ helpers
    def _check(self, what: str) -> None:
        code = int(_cuda().symm_status(True))
        if code:
            raise CommTimeout(f"device communicator: {what} gave up waiting for a peer (status {code})")

    def _stage_bytes(self, dst: torch.Tensor, data: bytes) -> None:
        if len(data) > self.cap:
            raise CommError(f"message of {len(data)} bytes exceeds the device communicator's {self.cap}")
        host = torch.empty(_HDR + len(data), dtype=torch.uint8).pin_memory()
        host[:8] = torch.tensor([len(data)], dtype=torch.int64).view(torch.uint8)
        host[8:_HDR] = 0
        if data:
            host[_HDR:] = torch.frombuffer(bytearray(data), dtype=torch.uint8)
        dst[:_HDR + len(data)].copy_(host, non_blocking=True)

    def _read_msgs(self, base: torch.Tensor, count: int) -> List[bytes]:
        """Messages in slots 0..count-1 of ``base`` (header + payload each) -> host bytes."""
        hdr = base.view(-1, self.slot)[:count, :8].contiguous().cpu()
        lens = hdr.view(torch.int64).reshape(-1).tolist()
        out = []
        for k, ln in enumerate(lens):
            if ln < 0 or ln > self.cap:
                raise CommError(f"device communicator: corrupt message length {ln}")
            lo = k * self.slot + _HDR
            out.append(bytes(base[lo:lo + ln].cpu().numpy().tobytes()) if ln else b"")
        return out

    def _barrier_slot(self, slot: int) -> None:
        _cuda().symm_barrier(self.ctx.flags.ptrs, self._rank, slot, self.epoch, 60 + slot)

    def _pull(self, data: Optional[bytes], peers: Sequence[int], stage: bool = True) -> List[bytes]:
        """Collective: stage ``data`` (when given), meet, pull the messages of ``peers``
        into inbox slots 0..len(peers)-1, meet again (the staging buffers may then be
        reused), return those messages."""
        self.epoch += 1
        if stage and data is not None:
            self._stage_bytes(self.stage.tensor, data)
        self._barrier_slot(0)
        if peers:
            _cuda().symm_pull_msgs(self.stage.ptrs, 0, self.inbox.data_ptr(), self.slot, list(peers),
                                   list(range(len(peers))), 4)
        self._barrier_slot(1)
        torch.cuda.current_stream(self.device).synchronize()
        self._check("collective")
        return self._read_msgs(self.inbox, len(peers)) if peers else []

    # ------------------------------------------------------------ Communicator
    def all_reduce(self, data: bytes, op=ReduceOp.Sum, dtype=DType.U64) -> bytes:
        self.epoch += 1
        self._stage_bytes(self.stage.tensor, data)
        self._barrier_slot(0)
        _cuda().symm_allreduce_msgs(self.stage.ptrs, 0, self.inbox.data_ptr(), _DT_CODE[dtype], _OP_CODE[op],
                                    self.cap, self.ctas)
        self._barrier_slot(1)
        torch.cuda.current_stream(self.device).synchronize()
        self._check("all_reduce")
        return self._read_msgs(self.inbox, 1)[0]

    def broadcast(self, data: bytes, root: int) -> bytes:
        return self._pull(data if self._rank == root else None, [root])[0]

    def all_gather(self, data: bytes) -> List[bytes]:
        return self._pull(data, list(range(self._world)))

    def exchange(self, data: bytes, peers: Sequence[int]) -> List[bytes]:
        """One-shot neighbour exchange (collective over the group): every rank stages
        its message once and pulls each listed peer's message."""
        if len(peers) > 16:
            return None
        return self._pull(data, [int(p) for p in peers])

    def send(self, data: bytes, dst: int) -> None:
        if dst == self._rank:
            raise CommError("send to self")
        n = self._world
        seq = self.sent[dst]
        self._stage_bytes(self.sendbuf, data)
        if seq >= self.ring:  # the receiver must have taken message seq - ring out of this slot
            _cuda().symm_flag(0, 0, self.pflags.tensor.data_ptr() + 4 * (n + dst), seq - self.ring + 1, 61)
        slot = (self._rank * self.ring + seq % self.ring) * self.slot
        _cuda().copy_async(self.mail.ptrs[dst] + slot, self.sendbuf.data_ptr(), _HDR + len(data))
        # publish: posted[me] in the receiver's flag area = seq + 1
        _cuda().symm_flag(self.pflags.ptrs[dst] + 4 * self._rank, seq + 1, 0, 0, 62)
        self.sent[dst] = seq + 1

    def recv(self, src: int) -> bytes:
        if src == self._rank:
            raise CommError("recv from self")
        n = self._world
        seq = self.recvd[src]
        _cuda().symm_flag(0, 0, self.pflags.tensor.data_ptr() + 4 * src, seq + 1, 63)
        torch.cuda.current_stream(self.device).synchronize()
        self._check("recv")
        lo = (src * self.ring + seq % self.ring) * self.slot
        msg = self._read_msgs(self.mail.tensor[lo:lo + self.slot], 1)[0]
        # acknowledge: acks[me] in the sender's flag area = seq + 1
        _cuda().symm_flag(self.pflags.ptrs[src] + 4 * (n + self._rank), seq + 1, 0, 0, 64)
        self.recvd[src] = seq + 1
        return msg

    def barrier(self) -> None:
        self._pull(None, [], stage=False)

    def rank(self) -> int:
        return self._rank

    def world_size(self) -> int:
        return self._world

    def backend(self) -> str:
        return "symm"

    # ------------------------------------------------------------ tensor API (device data)
    def _coll(self):
        if self.coll is None:
            raise CommError("the tensor interface needs tensor_bytes > 0")
        return self.coll

    def all_reduce_tensor(self, t: torch.Tensor) -> torch.Tensor:
        """In-place sum over ranks of an fp32 / bf16 device tensor (NVLS when the buffers
        have a multicast address, else the two-shot peer-memory kernel)."""
        c = self._coll()
        if t.dtype not in (torch.float32, torch.bfloat16):
            raise CommError("all_reduce_tensor: fp32 or bf16")
        flat = t.reshape(-1)
        vec = 16 // t.element_size()
        n = flat.numel()
        npad = (n + vec * self._world - 1) // (vec * self._world) * (vec * self._world)
        if npad * t.element_size() > c.buf.tensor.numel() * 4:
            raise CommError("all_reduce_tensor: tensor larger than the communicator's tensor buffer")
        view = c.buf.tensor.view(t.dtype)
        view[:n].copy_(flat)
        if npad > n:
            view[n:npad].zero_()
        out = c.all_reduce_nvls(npad, t.dtype) if c.nvls else c.all_reduce(npad, t.dtype)
        flat.copy_(out[:n])
        return t

    def all_gather_tensor(self, out: torch.Tensor, inp: torch.Tensor) -> torch.Tensor:
        """out = concatenation over ranks of ``inp`` (same shape everywhere)."""
        c = self._coll()
        nb = inp.numel() * inp.element_size()
        nb16 = _round16(nb)
        if nb16 * self._world > c.recv.tensor.numel() * 4:
            raise CommError("all_gather_tensor: larger than the communicator's tensor buffer")
        c.buf.tensor.view(torch.uint8)[:nb].copy_(inp.reshape(-1).view(torch.uint8))
        c.all_gather(nb16)
        src = c.recv.tensor.view(torch.uint8)[:nb16 * self._world].view(self._world, nb16)[:, :nb]
        out.reshape(self._world, -1).view(torch.uint8).copy_(src)
        return out

    def broadcast_tensor(self, t: torch.Tensor, root: int) -> torch.Tensor:
        c = self._coll()
        nb = t.numel() * t.element_size()
        nb16 = _round16(nb)
        u8 = c.buf.tensor.view(torch.uint8)
        if self._rank == root:
            u8[:nb].copy_(t.reshape(-1).view(torch.uint8))
        c.broadcast(nb16, root)
        t.reshape(-1).view(torch.uint8).copy_(u8[:nb])
        return t

    def exchange_neighbors_tensor(self, t: torch.Tensor, topology) -> List[torch.Tensor]:
        """Torus neighbour exchange of a device tensor (peer stores into each
        neighbour's receive slot, one kernel): returns the tensors received from the
        neighbours in ``neighbors()`` order (+x, -x, +y, -y, ...)."""
        from ..parallel.symm import halo_plan

        c = self._coll()
        nbr_rank, nbr_slot = halo_plan(topology, self._rank, self.device)
        k = nbr_rank.numel()
        nb = t.numel() * t.element_size()
        nb16 = _round16(nb)
        if nb16 * k > c.recv.tensor.numel() * 4:
            raise CommError("exchange_neighbors_tensor: larger than the communicator's tensor buffer")
        u8 = c.buf.tensor.view(torch.uint8)
        u8[:nb].copy_(t.reshape(-1).view(torch.uint8))
        c.halo(nb16, nbr_rank, nbr_slot)
        r8 = c.recv.tensor.view(torch.uint8)
        return [r8[j * nb16:j * nb16 + nb].clone().view(t.dtype).reshape(t.shape) for j in range(k)]


__all__ = ["SymmCommunicator"]
