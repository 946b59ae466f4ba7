#!/usr/bin/env python
"""Collective microbenchmark: NCCL (torch.distributed) against the fused NVLink
kernels of mtorus.parallel.symm, one process per GPU.

    torchrun --nproc-per-node 8 bench/collectives.py [--max-mb 1024] [--min-kb 4]

Operations: all-reduce (fp32, bf16, fp8 E4M3), broadcast, all-gather and the 2-D torus
(2 x N/2) nearest-neighbour halo exchange (NCCL: batched isend/irecv to the 4
neighbours; mtorus: direct peer stores into per-direction receive slots).
All-reduce and broadcast also run through NVLS when the fabric offers multicast
(``mtorus_nvls_*``: multimem.ld_reduce / multimem.st through the switch); the
FP8 all-reduce decodes peers' codes, sums in fp32 and re-encodes (NCCL: fp8
tensors where the installed NCCL supports them, else reported unsupported).
Message sizes are powers of two.  Each point is the median of CUDA-event timed
iterations (max over ranks); bus bandwidth uses the usual factors
(all-reduce 2(n-1)/n, all-gather (n-1)/n, broadcast 1, halo: bytes sent per
rank = 4 x message) and the roofline fraction is against 770 GB/s per
direction per GPU (measured NVLink peer copy).  Prints one JSON line per point.
"""
import argparse
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

LINK_GBS = 770.0


def timed(fn, iters, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    ts = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    ts.sort()
    t = torch.tensor([ts[len(ts) // 2]], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--min-kb", type=int, default=4)
    ap.add_argument("--max-mb", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--ops", default="allreduce_f32,allreduce_bf16,allreduce_fp8,broadcast,broadcast_scatter,"
                                      "allgather,halo")
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    from mtorus.core.topology import MeshTorusHybrid
    from mtorus.parallel.symm import SymmCollectives, halo_plan

    max_bytes = args.max_mb << 20
    col = SymmCollectives(f"cuda:{local}", max_bytes=max_bytes)
    g = torch.Generator(device="cuda").manual_seed(rank)
    col.buf.tensor.uniform_(-1, 1, generator=g)
    nccl_buf = torch.empty(max_bytes // 4, device="cuda").uniform_(-1, 1, generator=g)
    nccl_out = torch.empty(max_bytes // 4 * world if world <= 8 else 1, device="cuda") if max_bytes * world <= (8 << 30) else None
    topo = MeshTorusHybrid.new_2d(2, max(1, world // 2), 1) if world % 2 == 0 else MeshTorusHybrid.new_2d(world, 1, 1)
    nr, ns = halo_plan(topo, rank, "cuda")
    nbrs = [int(x) for x in nr.tolist()]
    halo_recv = torch.empty(4 * (max_bytes // 4), device="cuda")
    sizes = []
    b = args.min_kb << 10
    while b <= max_bytes:
        sizes.append(b)
        b *= 2
    for op in args.ops.split(","):
        for nbytes in sizes:
            f_v = None
            if op == "allreduce_f32":
                n = nbytes // 4
                f_n = lambda: dist.all_reduce(nccl_buf[:n])
                f_m = lambda: col.all_reduce(n, torch.float32)
                f_v = (lambda: col.all_reduce_nvls(n, torch.float32)) if col.nvls else None
                factor = 2 * (world - 1) / world
            elif op == "allreduce_bf16":
                n = nbytes // 2
                nb16 = nccl_buf.view(torch.bfloat16)
                f_n = lambda: dist.all_reduce(nb16[:n])
                f_m = lambda: col.all_reduce(n, torch.bfloat16)
                f_v = (lambda: col.all_reduce_nvls(n, torch.bfloat16)) if col.nvls else None
                factor = 2 * (world - 1) / world
            elif op == "allreduce_fp8":
                n = nbytes
                nb8 = nccl_buf.view(torch.uint8)[:n].view(torch.float8_e4m3fn)
                f_n = lambda: dist.all_reduce(nb8)
                f_m = lambda: col.all_reduce_fp8(n, 0)
                factor = 2 * (world - 1) / world
            elif op == "broadcast":
                n = nbytes // 4
                f_n = lambda: dist.broadcast(nccl_buf[:n], 0)
                f_m = lambda: col.broadcast(nbytes, 0)
                f_v = (lambda: col.broadcast_nvls(nbytes, 0)) if col.nvls else None
                factor = 1.0
            elif op == "broadcast_scatter":
                # scatter from the root by copy engine, then every rank multicasts its chunk
                if not col.nvls:
                    continue
                n = nbytes // 4
                f_n = lambda: dist.broadcast(nccl_buf[:n], 0)
                f_m = lambda: col.broadcast_scatter_nvls(nbytes, 0)
                factor = 1.0
            elif op == "allgather":
                if nbytes * world > max_bytes:
                    continue
                n = nbytes // 4
                f_n = lambda: dist.all_gather_into_tensor(nccl_out[:n * world], nccl_buf[:n])
                f_m = lambda: col.all_gather(nbytes)
                factor = (world - 1) / world * world  # bytes received per rank / message
            elif op == "halo":
                if 4 * nbytes > max_bytes:
                    continue
                n = nbytes // 4

                def f_n():
                    ops = []
                    for k, p in enumerate(nbrs):
                        ops.append(dist.P2POp(dist.isend, nccl_buf[:n], p))
                        ops.append(dist.P2POp(dist.irecv, halo_recv[k * n:(k + 1) * n], p))
                    for w in dist.batch_isend_irecv(ops):
                        w.wait()

                f_m = lambda: col.halo(nbytes, nr, ns)
                factor = len(nbrs)
            else:
                continue
            try:
                tn = timed(f_n, args.iters)
            except (RuntimeError, TypeError, ValueError) as e:  # dtype the NCCL build lacks
                tn = None
                nccl_err = str(e).splitlines()[0][:120]
            tm = timed(f_m, args.iters)
            tv = timed(f_v, args.iters) if f_v is not None else None
            bus = lambda t: nbytes * factor / (t * 1e-3) / 1e9  # noqa: E731
            if rank == 0:
                rec = {"op": op, "bytes": nbytes, "world": world,
                       "nccl_ms": round(tn, 4) if tn else None, "mtorus_ms": round(tm, 4),
                       "nccl_busbw_gbs": round(bus(tn), 1) if tn else None,
                       "mtorus_busbw_gbs": round(bus(tm), 1),
                       "mtorus_frac_of_link": round(bus(tm) / LINK_GBS, 3)}
                if tn is None:
                    rec["nccl"] = "unsupported: " + nccl_err
                if tv is not None:
                    rec.update({"mtorus_nvls_ms": round(tv, 4), "mtorus_nvls_busbw_gbs": round(bus(tv), 1),
                                "mtorus_nvls_frac_of_link": round(bus(tv) / LINK_GBS, 3)})
                rec["status"] = col.ctx.status(False)
                print(json.dumps(rec), flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
