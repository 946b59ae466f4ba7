"""Fused NVLink collectives over symmetric (peer-mapped) memory.

Buffers are allocated with torch's symmetric-memory allocator, which maps every
rank's allocation into every peer's address space (CUDA VMM + IPC handles on the
NVSwitch fabric); all data movement happens in the kernels of
``csrc/kernels/symm.cu`` with plain loads / stores to peer pointers and
epoch-stamped flags (bounded waits, no NCCL).

* ``SymmBucketReducer``  -- data-parallel gradient reduction: per 25 MB bucket, a
  reduce-scatter kernel (fp32 sum, 1/N averaging, Σg² and overflow flag fused)
  launched on a side stream as soon as backward finishes the bucket.
* ``ZeroAdam``           -- the sharded optimizer that consumes it: loss-scale /
  overflow / clip finalisation, Adam on this rank's shard, and the bf16 weight
  all-gather done by the same kernel storing each updated weight into every
  peer's weight buffer; a flag barrier then orders the next forward.
* ``SymmCollectives``    -- standalone all-reduce / all-gather / broadcast and the
  torus halo exchange for the collective microbenchmark.

Reference counterpart: the DP all-reduce primitive of crates/mt-comm/src/
collective.rs (never called by the reference's train_step) and the torus
neighbour exchange of crates/mt-comm/src/topology_aware.rs:38-49.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from ..ops.kernels import set_reserved_sms as _set_reserved_sms

from .._ext import cuda as _cuda
from .data_parallel import BucketPlan

_ALIGN = 64


def _group_name(group) -> str:
    g = group if group is not None else dist.group.WORLD
    return g.group_name


class SymmBuffer:
    """A symmetric allocation: the local tensor plus each peer's address of it."""

    def __init__(self, numel: int, dtype: torch.dtype, device, group=None, zero: bool = True):
        import torch.distributed._symmetric_memory as symm_mem

        self.tensor = symm_mem.empty(numel, dtype=dtype, device=device)
        if zero:
            self.tensor.zero_()
        self.handle = symm_mem.rendezvous(self.tensor, _group_name(group))
        self.rank = self.handle.rank
        self.world = self.handle.world_size
        base = self.handle.buffer_ptrs[self.rank]
        off = self.tensor.data_ptr() - base
        self.ptrs: List[int] = [int(p) + off for p in self.handle.buffer_ptrs]
        # NVLink multicast (NVLS) address of the same bytes, 0 when the fabric has none
        try:
            mc = int(self.handle.multicast_ptr)  # 0 when the allocation has no multicast binding
        except (AttributeError, RuntimeError):
            mc = 0
        self.mc = mc + off if mc else 0

    def barrier(self) -> None:
        self.handle.barrier()


class SymmContext:
    """Flag / scalar areas shared by the fused kernels of one process group."""

    def __init__(self, device, group=None, num_slots: int = 1024):
        self.device = torch.device(device)
        self.group = group
        self.flags = SymmBuffer(num_slots * 8, torch.int32, device, group)
        self.scalars = SymmBuffer(64, torch.float32, device, group)
        self.rank = self.flags.rank
        self.world = self.flags.world
        self.num_slots = num_slots
        # device-resident step counter: kernels given its address (ep_ptr) stamp and
        # wait on host epoch + counter, so a CUDA graph that advances it replays
        # every step with fresh epochs
        self.epoch_dev = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.ep_ptr = self.epoch_dev.data_ptr()
        self.flags.barrier()

    def advance_epoch(self) -> None:
        """+1 on the device step counter, in stream order on the current stream."""
        _cuda().symm_epoch_advance(self.epoch_dev)

    def status(self, reset: bool = True) -> int:
        """Non-zero when a fused kernel gave up waiting for a peer (its wait code)."""
        return int(_cuda().symm_status(reset))


def _mc_choice(env: str, world: int) -> bool:
    """A multicast (NVLS) variant: the environment variable forces it on ("1") or off ("0");
    unset, it is on from 4 ranks up."""
    import os

    v = os.environ.get(env)
    return v == "1" if v in ("0", "1") else world >= 4


def _chunk_len(n_elems: int, world: int) -> int:
    c = (n_elems + world - 1) // world
    return (c + _ALIGN - 1) // _ALIGN * _ALIGN


class SymmBucketReducer:
    """Reduce-scatter of the flat gradient buffer, bucket by bucket, over NVLink."""

    def __init__(self, flat, group=None, bucket_bytes: int = 25 * 1024 * 1024, ctas: Optional[int] = None,
                 ctx: Optional[SymmContext] = None, reserve_sms: Optional[int] = None,
                 grad_fp8: Optional[bool] = None):
        import os

        ctas = ctas if ctas is not None else int(os.environ.get("MTORUS_DP_CTAS", "16"))
        self.reserve = reserve_sms if reserve_sms is not None else int(os.environ.get("MTORUS_DP_RESERVE_SMS", str(ctas)))
        if not getattr(flat, "symmetric", False):
            raise ValueError("SymmBucketReducer needs a FlatParams built with symmetric grad/w16 buffers")
        self.flat = flat
        self.ctx = ctx or SymmContext(flat.device, group, num_slots=max(1024, 4 * (flat.numel // 1000000 + 8)))
        self.plan = BucketPlan(flat, bucket_bytes)
        nb = len(self.plan)
        if nb + 4 > self.ctx.num_slots:
            raise ValueError("too many buckets for the flag area")
        self.me, self.world = self.ctx.rank, self.ctx.world
        self.ctas = ctas
        # flags are stamped with the context's device step counter (advanced by
        # begin_step on the stream), so the step can be captured in a CUDA graph
        self.epoch = 0
        self.ep_ptr = self.ctx.ep_ptr
        self.stream = torch.cuda.Stream(priority=-1)
        self.slot_norm = nb
        self.slot_ag = nb + 1
        # this rank's shard: its chunk of every bucket -> (flat offset, len, compact offset)
        ranges, moff = [], 0
        self.clen = []
        for s, e in self.plan.ranges:
            c = _chunk_len(e - s, self.world)
            self.clen.append(c)
            c0 = s + self.me * c
            ln = max(0, min(e, c0 + c) - c0)
            if ln > 0:
                ranges.append((c0, ln, moff))
                moff += (ln + 7) // 8 * 8
        self.shard_numel = moff
        self.ranges = torch.tensor(ranges, dtype=torch.int64, device=flat.device).reshape(-1, 3)
        self._reserved = False
        # NVLS reduce-scatter (multimem.ld_reduce: the switch sums a chunk over all ranks, so each rank
        # receives its chunk once instead of n - 1 times) when the buffer has a multicast binding:
        # by default from 4 ranks up (with 2 the switch round trip buys nothing); MTORUS_DP_NVLS=1 / 0
        # forces it on / off
        self.nvls = _mc_choice("MTORUS_DP_NVLS", self.world) and self.flat.symm_grad.mc != 0
        # E5M2 gradient transport (opt-in): buckets cross NVLink as E5M2 codes with one
        # power-of-two scale per 32 values, decoded and summed in fp32 by the reduce kernel
        self.grad_fp8 = grad_fp8 if grad_fp8 is not None else os.environ.get("MTORUS_DP_GRAD_FP8") == "1"
        if self.grad_fp8:
            if flat.numel % 32:
                raise ValueError("E5M2 gradient transport needs a flat buffer of whole 32-value blocks")
            self.codes = SymmBuffer(flat.numel, torch.uint8, flat.device, group, zero=False)
            self.gsf = SymmBuffer(flat.numel // 32, torch.uint8, flat.device, group, zero=False)
        self._reset()

    def _reset(self):
        self.pending = [len(m) for m in self.plan.members]
        self.next_to_launch = 0

    def begin_step(self) -> None:
        """Start a step: advance the device step counter on the current stream
        (every rank takes the same number of steps, so the counters agree)."""
        self.ctx.advance_epoch()
        self._reserved = False

    def on_ready(self, params) -> None:
        for p in params:
            for q in getattr(p, "members", [p]):
                b = self.plan.bucket_of.get(id(q))
                if b is not None:
                    self.pending[b] -= 1
        while self.next_to_launch < len(self.plan) and self.pending[self.next_to_launch] <= 0:
            self._launch(self.next_to_launch)
            self.next_to_launch += 1

    def _launch(self, b: int) -> None:
        if not self._reserved:
            # from now on reduce kernels overlap backward: keep their SMs out of the GEMM grids
            _set_reserved_sms(self.reserve)
            self._reserved = True
        s, e = self.plan.ranges[b]
        ev = torch.cuda.Event()
        ev.record()
        self.stream.wait_event(ev)
        with torch.cuda.stream(self.stream):
            if self.grad_fp8:
                g = self.flat.symm_grad
                _cuda().dp_quant_e5m2(g.tensor.data_ptr() + 4 * s, self.codes.tensor.data_ptr() + s,
                                      self.gsf.tensor.data_ptr() + s // 32, e - s)
                _cuda().symm_rs_bucket_e5m2(self.codes.ptrs, self.gsf.ptrs, self.ctx.flags.ptrs, self.me, s, e - s,
                                            self.clen[b], b, self.epoch, self.state, self.ctas, 1.0 / self.world,
                                            g.tensor.data_ptr(), self.ep_ptr)
            elif self.nvls:
                _cuda().symm_rs_bucket_mc(self.flat.symm_grad.mc, self.flat.symm_grad.ptrs, self.ctx.flags.ptrs,
                                          self.me, s, e - s, self.clen[b], b, self.epoch, self.state, self.ctas,
                                          1.0 / self.world, self.ep_ptr)
            else:
                _cuda().symm_rs_bucket(self.flat.symm_grad.ptrs, self.ctx.flags.ptrs, self.me, s, e - s,
                                       self.clen[b], b, self.epoch, self.state, self.ctas, 1.0 / self.world,
                                       self.ep_ptr)

    def finish(self) -> None:
        while self.next_to_launch < len(self.plan):
            self._launch(self.next_to_launch)
            self.next_to_launch += 1
        with torch.cuda.stream(self.stream):
            _cuda().symm_scalars_ar(self.ctx.scalars.ptrs, self.ctx.flags.ptrs, self.me, self.slot_norm,
                                    self.epoch, self.state, self.ep_ptr)
        torch.cuda.current_stream().wait_stream(self.stream)
        _set_reserved_sms(0)
        self._reserved = False
        self._reset()

    # the optimizer's state block is shared (norm partials land in it)
    state: torch.Tensor = None


class ZeroAdam:
    """Adam over this rank's shard, fed by SymmBucketReducer; the new bf16 weights
    are written into every rank's weight buffer by the same kernel."""

    def __init__(self, flat, reducer: SymmBucketReducer, lr: float = 3e-4, betas=(0.9, 0.999), eps: float = 1e-5,
                 weight_decay: float = 0.0, max_grad_norm: float = 0.0, loss_scale=None):
        from ..training.fused_optim import ST_SCALE, DeviceLossScaleConfig

        self.flat = flat
        self.reducer = reducer
        self.lr = lr
        self.betas = betas
        self.eps = eps
        self.weight_decay = weight_decay
        self.max_grad_norm = max_grad_norm
        self.ls = loss_scale or DeviceLossScaleConfig()
        dev = flat.device
        self.m = torch.zeros(reducer.shard_numel, dtype=torch.float32, device=dev)
        self.v = torch.zeros_like(self.m)
        self.state = torch.zeros(16, dtype=torch.float32, device=dev)
        self.state[ST_SCALE] = self.ls.init_scale
        reducer.state = self.state
        # the new bf16 weights leave through the weight buffer's multicast address (one store,
        # replicated by the switch) when it has one: by default from 4 ranks up
        # (MTORUS_DP_AG_MC=1 / 0 forces it on / off)
        mc = flat.symm_w16.mc
        self.w16_mc = mc if mc and _mc_choice("MTORUS_DP_AG_MC", reducer.world) else 0

    @property
    def loss_scale_tensor(self) -> torch.Tensor:
        from ..training.fused_optim import ST_SCALE

        return self.state[ST_SCALE:ST_SCALE + 1]

    def finalize(self) -> None:
        """Overflow / loss-scale / clip decision from the norm partials the reduce
        kernels summed over the data-parallel ranks (a pipeline sums them over its
        stages first)."""
        from ..ops import kernels as K

        K.optim_finalize(self.state, self.ls.dynamic, self.ls.growth_interval, self.max_grad_norm, True)

    def step(self, lr: Optional[float] = None) -> None:
        self.finalize()
        self.update(lr)

    def update(self, lr: Optional[float] = None) -> None:
        """Adam on this rank's shard; the new bf16 weights go into every peer's weight
        buffer, then a flag barrier orders them before any rank's next forward."""
        r = self.reducer
        _cuda().symm_adam_shard_ag(r.ranges, self.flat.master, self.m, self.v, self.flat.grad,
                                   self.flat.symm_w16.ptrs, self.state, self.lr if lr is None else lr,
                                   self.betas[0], self.betas[1], self.eps, self.weight_decay, self.w16_mc)
        # every rank has written its shard into every peer: order the next forward after it
        _cuda().symm_barrier(r.ctx.flags.ptrs, r.me, r.slot_ag, r.epoch, 23, r.ep_ptr)

    def stats(self) -> dict:
        s = self.state.tolist()
        return {"loss_scale": s[2], "grad_norm": s[6], "skipped": s[5] > 0, "steps": int(s[7])}


class SymmCollectives:
    """Standalone NVLink collectives on symmetric buffers (microbenchmark / halo)."""

    def __init__(self, device, group=None, max_bytes: int = 1 << 30, ctas: int = 128):
        self.ctx = SymmContext(device, group)
        self.me, self.world = self.ctx.rank, self.ctx.world
        self.buf = SymmBuffer(max_bytes // 4, torch.float32, device, group)
        self.recv = SymmBuffer(max_bytes // 4, torch.float32, device, group)
        self.ctas = ctas
        self.epoch = 0

    def _slot(self):
        self.epoch += 1
        return self.epoch

    def all_reduce(self, numel: int, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """In-place sum over ranks of the first numel elements of ``buf`` (as dtype)."""
        ep = self._slot()
        _cuda().symm_allreduce(self.buf.ptrs, self.ctx.flags.ptrs, self.me, numel, 0 if dtype == torch.float32 else 1,
                               0, ep, self.ctas)
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 1, ep, 32)
        return self.buf.tensor.view(dtype)[:numel]

    @property
    def nvls(self) -> bool:
        """True when the buffers have an NVLink multicast address (NVSwitch reduction)."""
        return self.buf.mc != 0

    def all_reduce_nvls(self, numel: int, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """In-place sum over ranks through NVLS: each rank reduces its slice in the
        switch (multimem.ld_reduce) and stores it to every rank (multimem.st)."""
        ep = self._slot()
        _cuda().symm_allreduce_mc(self.buf.mc, self.buf.ptrs, self.ctx.flags.ptrs, self.me, numel,
                                  0 if dtype == torch.float32 else 1, 6, ep, self.ctas)
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 7, ep, 37)
        return self.buf.tensor.view(dtype)[:numel]

    def all_reduce_fp8(self, numel: int, fmt: int = 0) -> torch.Tensor:
        """In-place sum over ranks of ``numel`` FP8 codes (0: E4M3, 1: E5M2): fp32
        accumulation, saturating re-encode, result in every rank's buffer."""
        ep = self._slot()
        _cuda().symm_allreduce_mc(0, self.buf.ptrs, self.ctx.flags.ptrs, self.me, numel, 2 + fmt, 8, ep, self.ctas)
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 9, ep, 38)
        return self.buf.tensor.view(torch.uint8)[:numel]

    def broadcast_nvls(self, nbytes: int, root: int = 0) -> None:
        """The root stores its bytes once into the multicast address; the switch
        writes every rank's copy."""
        ep = self._slot()
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 10, ep, 39)  # every rank is past its last read
        if self.me == root:
            _cuda().symm_broadcast_mc(self.buf.tensor.data_ptr(), self.buf.mc, nbytes, self.ctas)
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 11, ep, 40)

    def broadcast_scatter_nvls(self, nbytes: int, root: int = 0) -> None:
        """Broadcast as scatter + multicast: the root's copy engine sends chunk p of its
        bytes to rank p (one ``cudaMemcpyAsync`` per peer over NVLink), then every rank
        stores its chunk once into the multicast address (``multimem.st``) and the
        switch writes it into every rank's buffer.  The root's link carries (n-1)/n of
        the bytes once and the multicast stores run on all ranks at the same time,
        instead of one GPU issuing every multicast store (``broadcast_nvls``)."""
        if nbytes % 16:
            raise ValueError("broadcast_scatter_nvls: nbytes must be a multiple of 16")
        n = self.world
        chunk = ((nbytes + n - 1) // n + 15) // 16 * 16
        ep = self._slot()
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 12, ep, 41)  # every rank is past its last read
        if self.me == root:
            base = self.buf.tensor.data_ptr()
            for p in range(n):
                lo = min(nbytes, p * chunk)
                ln = min(nbytes, lo + chunk) - lo
                if p != root and ln > 0:
                    _cuda().copy_async(self.buf.ptrs[p] + lo, base + lo, ln)
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 13, ep, 42)  # chunk me has landed here
        lo = min(nbytes, self.me * chunk)
        ln = min(nbytes, lo + chunk) - lo
        if ln > 0:
            _cuda().symm_broadcast_mc(self.buf.tensor.data_ptr() + lo, self.buf.mc + lo, ln, self.ctas)
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 14, ep, 43)

    def all_gather(self, nbytes: int) -> None:
        """Each rank's first nbytes of ``buf`` land in slot rank of every peer's ``recv``."""
        ep = self._slot()
        _cuda().symm_allgather(self.buf.tensor.data_ptr(), self.recv.ptrs, self.me, nbytes, self.ctas)
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 2, ep, 33)

    def broadcast(self, nbytes: int, root: int = 0) -> None:
        ep = self._slot()
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 3, ep, 34)  # root's data is ready everywhere
        if self.me == root:
            _cuda().symm_broadcast(self.buf.ptrs, root, nbytes, self.ctas)
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 4, ep, 35)

    def halo(self, nbytes: int, nbr_rank: torch.Tensor, nbr_slot: torch.Tensor) -> None:
        """Store ``buf[:nbytes]`` into slot nbr_slot[k] of neighbour nbr_rank[k]'s ``recv``."""
        ep = self._slot()
        _cuda().symm_halo(self.buf.tensor.data_ptr(), self.recv.ptrs, nbr_rank, nbr_slot, nbytes, self.ctas)
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 5, ep, 36)


class GatheredOperand:
    """An FP8 GEMM operand sharded by rows over the ranks of a group and read by the
    GEMM straight from its owners: the parameter all-gather fused into the first GEMM
    that consumes the parameters (``gemm_fp8_gather_b``).

    The reference gathers with a blocking ``all_gather`` of whole byte buffers
    (crates/mt-comm/src/topology_aware.rs:58-66).  Here each rank writes only its own
    rows, ``[rank * shard_rows, (rank + 1) * shard_rows)``, into a symmetric buffer
    (``local_shard()``), ``publish()`` orders those writes before any peer's read
    (a barrier over the ranks), and a GEMM then reads the remote rows in one of two
    ways:

    * ``direct``: the GEMM's TMA producer loads each 128-row (K-major) or 128-deep
      (MN-major) tile from the rank that owns it, over NVLink, with plain (never
      multicast) loads.  Peer reads are cached in the owner's L2, not this GPU's, so
      every output row block re-reads the remote tiles: right for small M (one or two
      256-row blocks, e.g. a decode step), NVLink-bound for training-sized M.
    * ``overlap``: shard by shard, starting with the own one, the GEMM runs on the
      shards already local while the copy engine pulls the next shard from its owner
      (one ``cudaMemcpyAsync`` per shard on a side stream): every remote byte crosses
      NVLink once and the copies hide behind the math.

    ``method="auto"`` picks ``direct`` when M spans at most two 256-row blocks.
    shard_rows is rounded up to 128 so that no tile spans two owners.  A rank must
    not rewrite its shard before every rank finished the GEMMs that read it
    (``retire()``).
    """

    def __init__(self, rows: int, cols: int, device, group=None, ctx: "SymmContext" = None):
        if cols % 16:
            raise ValueError("GatheredOperand: cols must be a multiple of 16 (TMA row stride)")
        self.ctx = ctx or SymmContext(device, group, num_slots=16)
        self.me, self.world = self.ctx.rank, self.ctx.world
        self.rows, self.cols = rows, cols
        per = (rows + self.world - 1) // self.world
        self.shard_rows = (per + 127) // 128 * 128
        self.buf = SymmBuffer(self.shard_rows * self.world * cols, torch.uint8, device, group)
        self.full = self.buf.tensor.view(self.shard_rows * self.world, cols)[:rows]
        self.lo = min(rows, self.me * self.shard_rows)
        self.hi = min(rows, self.lo + self.shard_rows)
        self.epoch = 0
        self.retired = 0
        self._gathered: Optional[torch.Tensor] = None
        self._copy_stream: Optional[torch.cuda.Stream] = None

    def shard_range(self, p: int):
        lo = min(self.rows, p * self.shard_rows)
        return lo, min(self.rows, lo + self.shard_rows)

    def local_shard(self) -> torch.Tensor:
        """This rank's rows of the operand (uint8 codes) to write into."""
        return self.full[self.lo:self.hi]

    def publish(self) -> None:
        """Every rank's shard writes (stream-ordered before this call) become visible
        to all ranks' later GEMMs.  Call on every rank."""
        self.epoch += 1
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 0, self.epoch, 44)

    def retire(self) -> None:
        """Every rank's GEMMs on the current shards are done (stream order), so owners
        may rewrite them.  Call on every rank."""
        self.retired += 1
        _cuda().symm_barrier(self.ctx.flags.ptrs, self.me, 1, self.retired, 45)

    def gemm(self, a: torch.Tensor, a_fmt: int, b_fmt: int, out: Optional[torch.Tensor] = None, *,
             a_mn: bool = False, b_mn: bool = False, bias=None, residual=None, act=None, aux=None, alpha=None,
             alpha2=None, accumulate: bool = False, out_dtype: torch.dtype = torch.bfloat16,
             method: str = "auto") -> torch.Tensor:
        """out = epilogue(alpha * alpha2 * A . B^T) with B this operand: [N, K] = [rows, cols]
        (b_mn=False) or [K, N] = [rows, cols] (b_mn=True, rows sharded along K)."""
        M = a.shape[1] if a_mn else a.shape[0]
        N = self.cols if b_mn else self.rows
        if out is None:
            out = torch.empty((M, N), dtype=out_dtype, device=a.device)
        if method == "auto":
            method = "direct" if (M + 255) // 256 <= 2 else "overlap"
        if method == "direct":
            _cuda().gemm_fp8_gather_b(a, bool(a_mn), int(a_fmt), self.full, bool(b_mn), int(b_fmt), self.buf.ptrs,
                                      self.shard_rows, out, bias, residual, act, aux, alpha, alpha2,
                                      bool(accumulate))
            return out
        if method != "overlap":
            raise ValueError(f"method must be auto, direct or overlap, not {method!r}")
        return self._gemm_overlap(a, a_fmt, b_fmt, out, a_mn, b_mn, bias, residual, act, aux, alpha, alpha2,
                                  accumulate)

    def _gemm_overlap(self, a, a_fmt, b_fmt, out, a_mn, b_mn, bias, residual, act, aux, alpha, alpha2, accumulate):
        from ..ops.fp8 import gemm_fp8

        if b_mn and (out.dtype != torch.float32 or any(t is not None for t in (bias, residual, act, aux))):
            raise ValueError("overlap with a K-sharded B sums per-shard partial products: fp32 output, "
                             "no bias / residual / GELU epilogue")
        cur = torch.cuda.current_stream()
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(device=a.device)
            self._gathered = torch.empty((self.rows, self.cols), dtype=torch.uint8, device=a.device)
        cs, g = self._copy_stream, self._gathered
        order = [(self.me + i) % self.world for i in range(self.world)]
        ready = {}
        cs.wait_stream(cur)  # the owners' writes were published on this stream
        with torch.cuda.stream(cs):
            for p in order[1:]:
                lo, hi = self.shard_range(p)
                if hi > lo:
                    _cuda().copy_async(g[lo:hi].data_ptr(), self.buf.ptrs[p] + lo * self.cols, (hi - lo) * self.cols)
                ev = torch.cuda.Event()
                ev.record(cs)
                ready[p] = ev
        first = True
        for p in order:
            lo, hi = self.shard_range(p)
            if hi <= lo:
                continue
            if p != self.me:
                cur.wait_event(ready[p])
            src = (self.full if p == self.me else g)[lo:hi]
            if not b_mn:  # this shard's rows of B are output columns lo..hi
                sl = (slice(None), slice(lo, hi))
                gemm_fp8(a, a_fmt, src, b_fmt, out[sl], a_mn=a_mn, alpha=alpha, alpha2=alpha2,
                         bias=None if bias is None else bias[lo:hi],
                         residual=None if residual is None else residual[sl], act=None if act is None else act[sl],
                         aux=None if aux is None else aux[sl], accumulate=accumulate)
            else:  # this shard is K rows lo..hi: add its partial product
                a_k = a[lo:hi] if a_mn else a[:, lo:hi]
                gemm_fp8(a_k, a_fmt, src, b_fmt, out, a_mn=a_mn, b_mn=True, alpha=alpha, alpha2=alpha2,
                         accumulate=accumulate or not first)
            first = False
        cs.wait_stream(cur)  # the gathered copy stays untouched until these GEMMs ran
        return out


def halo_plan(topology, rank: int, device) -> tuple:
    """Neighbour ranks and receive slots for the torus exchange of ``rank``: the
    sender's k-th neighbour (+x, -x, +y, -y, ...) receives into its slot for the
    opposite direction, so a 2-wide axis (where +x == -x) keeps both messages."""
    coords = topology.rank_to_coords(rank)
    nbrs = coords.neighbors(topology.dims)
    ranks, slots = [], []
    for k, (c, axis) in enumerate(nbrs):
        ranks.append(topology.node_rank(c))
        slots.append(k ^ 1)  # +axis send arrives in the receiver's -axis slot
    return (torch.tensor(ranks, dtype=torch.int32, device=device),
            torch.tensor(slots, dtype=torch.int32, device=device))


__all__ = ["SymmBuffer", "SymmContext", "SymmBucketReducer", "ZeroAdam", "SymmCollectives", "GatheredOperand",
           "halo_plan"]
