#!/usr/bin/env python
"""Weight all-gather fused into the FP8 GEMM that consumes the weights, against the NCCL baseline.

Each rank owns 1/N of the rows of an E4M3 weight W [N_out, K] (the GPT-1B FFN1
weight: 8192 x 2048) and computes Y = X . W^T for its own activations X [M, K]:

* ``nccl``    -- all_gather_into_tensor of the shards, then the tcgen05 FP8 GEMM;
* ``overlap`` -- GatheredOperand, the GEMM on the shards already local while the
                 copy engine pulls the next one from its owner;
* ``direct``  -- GatheredOperand, the GEMM's TMA producer reads remote tiles from
                 their owners (no gathered copy; for small M).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 bench/gather_gemm_bench.py --m 16384 256

Times each variant with CUDA events (median of --iters after warm-up), max over
ranks, and prints one JSON line per (M, variant) on rank 0 with the roofline: the
slower of the GEMM at the FP8 peak (2x the measured bf16 cuBLAS figure) and the
remote weight bytes over NVLink at 770 GB/s per direction (measured peer copy).
"""
import argparse
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, nargs="+", default=[16384, 256])
    ap.add_argument("--n-out", type=int, default=8192)
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    args = ap.parse_args()
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from mtorus.ops import fp8 as F8
    from mtorus.parallel.symm import GatheredOperand

    peak = 1607.9
    pk = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        peak = json.load(open(pk)).get("bf16_tflops", peak)
    N, K = args.n_out, args.k
    w = GatheredOperand(N, K, dev)
    g = torch.Generator(device=dev).manual_seed(1 + rank)
    w.local_shard().copy_((torch.randn(w.hi - w.lo, K, device=dev, generator=g) * 0.1).to(torch.float8_e4m3fn)
                          .view(torch.uint8))
    w.publish()
    shard = w.local_shard().contiguous()
    rows_pad = w.shard_rows * world
    gathered = torch.empty(rows_pad, K, dtype=torch.uint8, device=dev)
    pad = torch.zeros(w.shard_rows, K, dtype=torch.uint8, device=dev)
    pad[: shard.shape[0]] = shard
    one = torch.ones(1, device=dev)

    def nccl_variant(x):
        dist.all_gather_into_tensor(gathered, pad)
        return F8.gemm_fp8(x, 0, gathered[:N], 0, alpha=one)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        ts = []
        for _ in range(args.iters):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b))
        ts.sort()
        t = torch.tensor([ts[len(ts) // 2]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    for M in args.m:
        x = (torch.randn(M, K, device=dev, generator=g)).to(torch.float8_e4m3fn).view(torch.uint8)
        flops = 2.0 * M * N * K
        remote = (world - 1) / world * N * K  # weight bytes that must cross NVLink into this GPU
        roof_ms = max(flops / (2 * peak * 1e12), remote / 770e9) * 1e3
        variants = {"nccl": lambda: nccl_variant(x),
                    "overlap": lambda: w.gemm(x, 0, 0, alpha=one, method="overlap"),
                    "direct": lambda: w.gemm(x, 0, 0, alpha=one, method="direct")}
        for name, fn in variants.items():
            ms = timed(fn)
            if rank == 0:
                print(json.dumps({"bench": "allgather_gemm_fp8", "variant": name, "n_gpus": world, "M": M, "N": N,
                                  "K": K, "ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1),
                                  "roofline_ms": round(roof_ms, 4), "frac_of_roofline": round(roof_ms / ms, 3)}),
                      flush=True)
        w.retire()
    torch.cuda.synchronize()
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
