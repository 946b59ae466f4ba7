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
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist


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


class NcclBucketReducer:
    """Averages gradients across the DP group with NCCL, overlapped with backward."""

    def __init__(self, flat, group=None, bucket_bytes: int = 25 * 1024 * 1024, reserve_sms: Optional[int] = None):
        import os

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
            from .._ext import cuda as _cuda

            _cuda().gemm_set_reserved_sms(self.reserve_sms)
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
        dist.all_reduce(self.flat.grad[s:e], op=dist.ReduceOp.AVG, group=self.group)

    def finish(self) -> None:
        while self.next_to_launch < len(self.plan):
            self._launch(self.next_to_launch)
            self.next_to_launch += 1
        if self.on_cuda:
            torch.cuda.current_stream().wait_stream(self.stream)
            if self.reserve_sms:
                from .._ext import cuda as _cuda

                _cuda().gemm_set_reserved_sms(0)
        self._reset()
