#!/usr/bin/env python
"""FP8 quantise kernel with and without the fused amax all-reduce (the amax is
published to every rank by the last block of each quantise kernel).

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 bench/fp8_quant_bench.py

Per rank: a [16384, 8192] bf16 tensor (268 MB, larger than L2) quantised to E4M3
with the delayed scale: plain kernel (local amax only) vs the kernel whose last
block publishes the amax into every peer's table over NVLink.  Device-timed with
CUDA events, max over ranks; bytes = 2n read + n written; roofline = measured
HBM copy bandwidth (MEASURED_PEAKS.json).  Rank 0 prints one JSON line per case.
"""
import json
import os
import sys
from datetime import timedelta

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from mtorus.ops import fp8 as F8

    hbm = 6526.2
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    if os.path.exists(p):
        hbm = json.load(open(p)).get("hbm_gbs", hbm)
    x = torch.randn(16384, 8192, device=dev).bfloat16()
    out = torch.empty(x.shape, dtype=torch.uint8, device=dev)
    st = F8.Fp8State(dev, history=16, capacity=64)
    sync = F8.SymmAmaxSync(dev, st.cap)
    slot = st.slot("x", F8.E4M3)
    sl = slice(slot, slot + 1)
    cases = {
        "quantize_local_amax": lambda: F8.quantize(x, F8.E4M3, st.scale[sl], st.amax[sl], out=out),
        "quantize_fused_amax_allreduce": lambda: sync.quantize(x, out, st.scale[sl], st.amax[sl], slot, F8.E4M3),
    }
    iters = 20
    for name, fn in cases.items():
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        b.synchronize()
        ms = torch.tensor([a.elapsed_time(b) / iters], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        ms = float(ms)
        nbytes = 3 * x.numel()
        if rank == 0:
            print(json.dumps({"case": name, "world": world, "numel": x.numel(), "ms": round(ms, 4),
                              "gbs": round(nbytes / ms / 1e6, 1), "frac_of_measured_hbm": round(nbytes / ms / 1e6 / hbm, 3),
                              "nvlink_bytes_per_launch": 8 * world if "fused" in name else 0}), flush=True)
    sync.reduce(st.amax[:1])
    torch.cuda.synchronize()
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
