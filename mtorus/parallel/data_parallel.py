"""Data-parallel gradient reduction over the flat gradient buffer.

Buckets are contiguous ranges of the flat buffer, ~25 MB each, built back to
front because gradients become final in reverse layer order.  The fused
backward functions report finished parameters through
``FusedGradState.grad_ready_hook``; a bucket whose parameters are all final is
reduced on a dedicated communication stream while backward keeps running on
the compute stream.  Every rank launches buckets in the same (index) order.

Two reducers share this scheduling:

* ``NcclBucketReducer`` -- ``torch.distributed`` all-reduce (NCCL), the baseline;
* ``mtorus.parallel.symm.SymmBucketReducer`` -- the fused NVLink path.

Both can move the gradients as E5M2 with one power-of-two scale per 32 values
instead of fp32 (opt-in, ``grad_fp8=True`` or ``MTORUS_DP_GRAD_FP8=1``).  Here that
is an all-to-all of the encoded chunks (rank p receives chunk p of every rank's
bucket), an fp32 decode-and-average of the own chunk, and an all-gather of the
averaged chunks in bf16: about 3 bytes per gradient per rank on the wire instead of
the ~8 of an fp32 ring all-reduce, and every rank ends with identical values.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from ..ops.kernels import set_reserved_sms as _set_reserved_sms


class BucketPlan:
    def __init__(self, flat, bucket_bytes: int = 25 * 1024 * 1024, align_elems: int = 64):
        esize = flat.grad.element_size()
        cap = max(1, bucket_bytes // esize)
        params = sorted(flat.params, key=lambda p: p.flat_offset)
        self.ranges: List[List[int]] = []
        self.members: List[List[torch.nn.Parameter]] = []
        self.bucket_of = {}
        end = flat.numel
        cur: List[torch.nn.Parameter] = []
        cur_start = end
        for p in reversed(params):
            cur.append(p)
            cur_start = p.flat_offset
            if end - cur_start >= cap and cur_start % align_elems == 0:
                self._close(cur, cur_start, end, align_elems)
                end = self.ranges[-1][0]
                cur = []
        if cur:
            self._close(cur, 0, end, align_elems)
        # the first bucket must start at 0
        self.ranges[-1][0] = 0
        for b, ms in enumerate(self.members):
            for p in ms:
                self.bucket_of[id(p)] = b

    def _close(self, params, start, end, align):
        self.ranges.append([start, end])
        self.members.append(list(params))

    def __len__(self):
        return len(self.ranges)


E5M2_MAX = 57344.0  # largest finite E5M2 value


def e5m2_encode(x: torch.Tensor):
    """fp32 1-D (length a multiple of 32) -> (E5M2 codes uint8 [L], scale bytes uint8 [L / 32]):
    per 32-value block the smallest power of two that keeps the block's amax within the
    E5M2 range (UE8M0 byte X + 127; 255 marks a block with a NaN / Inf).  The CUDA
    kernel on the GPU, the PyTorch oracle on the CPU (identical rule and rounding)."""
    L = x.numel()
    if L % 32:
        raise ValueError("e5m2_encode: length must be a multiple of 32")
    if x.is_cuda:
        from .._ext import cuda as _cuda

        x = x.contiguous()
        codes = torch.empty(L, dtype=torch.uint8, device=x.device)
        sf = torch.empty(L // 32, dtype=torch.uint8, device=x.device)
        _cuda().dp_quant_e5m2(x.data_ptr(), codes.data_ptr(), sf.data_ptr(), L)
        return codes, sf
    from ..ops.mxfp8 import E5M2, mx_quantize_ref, sf_offsets

    t = mx_quantize_ref(x.reshape(-1, 32).float(), E5M2, E5M2_MAX)
    return t.codes.reshape(-1), t.sf[sf_offsets(L // 32, 32).reshape(-1)]


def e5m2_decode(codes: torch.Tensor, sf: torch.Tensor) -> torch.Tensor:
    """Inverse of ``e5m2_encode`` on the last dimension (fp32; NaN where the scale is 255)."""
    vals = codes.view(torch.float8_e5m2).float()
    b = sf.to(torch.int32)
    scale = torch.ldexp(torch.ones(b.shape, device=b.device), (b - 127).float())
    scale = torch.where(b == 255, torch.full_like(scale, float("nan")), scale)
    shape = vals.shape
    return (vals.reshape(*shape[:-1], -1, 32) * scale[..., None]).reshape(shape)


def _chunk(n_elems: int, world: int, align: int = 64) -> int:
    c = (n_elems + world - 1) // world
    return (c + align - 1) // align * align


class NcclBucketReducer:
    """Averages gradients across the DP group with NCCL, overlapped with backward."""

    def __init__(self, flat, group=None, bucket_bytes: int = 25 * 1024 * 1024, reserve_sms: Optional[int] = None,
                 grad_fp8: Optional[bool] = None):
        import os

        self.grad_fp8 = grad_fp8 if grad_fp8 is not None else os.environ.get("MTORUS_DP_GRAD_FP8") == "1"
        self.flat = flat
        self.group = group
        self.reserve_sms = reserve_sms if reserve_sms is not None else int(os.environ.get("MTORUS_DP_RESERVE_SMS", "16"))
        self.world = dist.get_world_size(group)
        self.plan = BucketPlan(flat, bucket_bytes)
        self.on_cuda = flat.grad.is_cuda
        self.stream = torch.cuda.Stream(priority=-1) if self.on_cuda else None
        self._reset()

    def _reset(self):
        self.pending = [len(m) for m in self.plan.members]
        self.launched = [False] * len(self.plan)
        self.next_to_launch = 0

    def on_ready(self, params) -> None:
        for p in params:
            for q in getattr(p, "members", [p]):
                b = self.plan.bucket_of.get(id(q))
                if b is not None:
                    self.pending[b] -= 1
        # launch in index order only (identical order on every rank)
        while self.next_to_launch < len(self.plan) and self.pending[self.next_to_launch] <= 0:
            self._launch(self.next_to_launch)
            self.next_to_launch += 1

    def _launch(self, b: int) -> None:
        s, e = self.plan.ranges[b]
        if self.on_cuda and b == 0 and self.reserve_sms:
            # NCCL kernels overlap the rest of backward: leave SMs free for them
            _set_reserved_sms(self.reserve_sms)
        if not self.on_cuda:
            self.reduce_range(s, e)
            self.launched[b] = True
            return
        ev = torch.cuda.Event()
        ev.record()
        self.stream.wait_event(ev)
        with torch.cuda.stream(self.stream):
            self.reduce_range(s, e)
        self.launched[b] = True

    def reduce_range(self, s: int, e: int) -> None:
        if self.grad_fp8:
            self._reduce_range_e5m2(s, e)
            return
        dist.all_reduce(self.flat.grad[s:e], op=dist.ReduceOp.AVG, group=self.group)

    def _reduce_range_e5m2(self, s: int, e: int) -> None:
        g = self.flat.grad[s:e]
        n, L = self.world, e - s
        c = _chunk(L, n)
        padded = torch.zeros(n * c, dtype=torch.float32, device=g.device)
        padded[:L] = g
        codes, sf = e5m2_encode(padded)
        rc = torch.empty(n, c, dtype=torch.uint8, device=g.device)
        rs = torch.empty(n, c // 32, dtype=torch.uint8, device=g.device)
        dist.all_to_all_single(rc, codes.view(n, c), group=self.group)  # row p: my chunk of rank p's bucket
        dist.all_to_all_single(rs, sf.view(n, c // 32), group=self.group)
        if g.is_cuda:
            from .._ext import cuda as _cuda

            mine = torch.empty(c, dtype=torch.bfloat16, device=g.device)
            _cuda().dp_decode_mean_e5m2(rc, rs, mine)  # decode, fp32 sum in rank order, scale, bf16
        else:
            mine = (e5m2_decode(rc, rs).sum(0) * (1.0 / n)).to(torch.bfloat16)
        gathered = torch.empty(n, c, dtype=torch.bfloat16, device=g.device)
        if g.is_cuda:
            dist.all_gather_into_tensor(gathered, mine, group=self.group)
        else:  # gloo: list form, bf16 carried as bytes
            parts = [torch.empty(2 * c, dtype=torch.uint8) for _ in range(n)]
            dist.all_gather(parts, mine.view(torch.uint8), group=self.group)
            gathered = torch.stack([t.view(torch.bfloat16) for t in parts])
        g.copy_(gathered.reshape(-1)[:L])

    def finish(self) -> None:
        while self.next_to_launch < len(self.plan):
            self._launch(self.next_to_launch)
            self.next_to_launch += 1
        if self.on_cuda:
            torch.cuda.current_stream().wait_stream(self.stream)
            if self.reserve_sms:
                _set_reserved_sms(0)
        self._reset()
