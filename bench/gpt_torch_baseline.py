#!/usr/bin/env python
"""Plain-PyTorch baseline for the GPT-1B training benchmark: the same model shape
and step in eager PyTorch -- nn.Linear / nn.LayerNorm (cuBLAS bf16 under autocast),
scaled_dot_product_attention (cuDNN / flash), torch.optim.Adam(fused=True), and
DistributedDataParallel with 25 MB buckets over NCCL for N > 1.  None of this
framework's kernels run on this path; it is the "PyTorch eager + cuBLAS + NCCL"
comparison point for ``bench.py``.  With ``--mx`` every Linear runs instead on mtorus'
MXFP8 recipe (``enable_mx_linears``): the same eager model with only the GEMMs swapped.

    python bench/gpt_torch_baseline.py --steps 10 --warmup 3
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 bench/gpt_torch_baseline.py

Prints one JSON line (rank 0): tokens/s over all GPUs, device-timed with CUDA
events, max over ranks.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
from datetime import timedelta

import torch
import torch.nn as nn
import torch.nn.functional as F


class Block(nn.Module):
    def __init__(self, d, h, f):
        super().__init__()
        self.h = h
        self.ln1, self.ln2 = nn.LayerNorm(d), nn.LayerNorm(d)
        self.qkv, self.proj = nn.Linear(d, 3 * d), nn.Linear(d, d)
        self.fc1, self.fc2 = nn.Linear(d, f), nn.Linear(f, d)

    def forward(self, x):
        B, S, d = x.shape
        q, k, v = self.qkv(self.ln1(x)).view(B, S, 3, self.h, d // self.h).unbind(2)
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True)
        x = x + self.proj(o.transpose(1, 2).reshape(B, S, d))
        return x + self.fc2(F.gelu(self.fc1(self.ln2(x))))


class GPT(nn.Module):
    def __init__(self, V, d, L, h, f, S):
        super().__init__()
        self.tok, self.pos = nn.Embedding(V, d), nn.Embedding(S, d)
        self.blocks = nn.ModuleList([Block(d, h, f) for _ in range(L)])
        self.ln_f, self.head = nn.LayerNorm(d), nn.Linear(d, V)
        for p in self.parameters():
            if p.dim() > 1:
                nn.init.normal_(p, 0.0, 0.02)

    def forward(self, ids):
        x = self.tok(ids) + self.pos(torch.arange(ids.shape[1], device=ids.device))
        for b in self.blocks:
            x = b(x)
        return self.head(self.ln_f(x))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--micro-batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--mx", action="store_true",
                    help="run every Linear through mtorus' MXFP8 recipe (block-scaled tcgen05 GEMMs) instead of "
                         "cuBLAS bf16: the eager model with only the GEMMs swapped")
    args = ap.parse_args()
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    V, d, h, f, S, B = 50304, 2048, 16, 8192, args.seq, args.micro_batch
    torch.manual_seed(1234)
    model = GPT(V, d, args.layers, h, f, S).to(dev)
    if args.mx:
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        from mtorus.ops.mxfp8 import enable_mx_linears

        enable_mx_linears(model)
    if world > 1:
        model = nn.parallel.DistributedDataParallel(model, device_ids=[local], bucket_cap_mb=25,
                                                    gradient_as_bucket_view=True)
    opt = torch.optim.Adam(model.parameters(), lr=3e-4, fused=True)
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    data = [torch.randint(0, V, (B, S + 1), device=dev, generator=gen) for _ in range(4)]

    def step(t):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = model(t[:, :-1])
            loss = F.cross_entropy(logits.float().view(-1, V), t[:, 1:].reshape(-1))
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss.detach()

    for i in range(args.warmup):
        step(data[i % 4])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[local])
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(args.steps):
        loss = step(data[i % 4])
    b.record()
    b.synchronize()
    ms = torch.tensor([a.elapsed_time(b) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms)
    nparams = sum(p.numel() for p in model.parameters())
    out = {"metric": ("GPT-1B MXFP8-linear tokens/sec, PyTorch eager with mtorus block-scaled GEMMs" if args.mx else
                      "GPT-1B bf16 tokens/sec, plain PyTorch eager (cuBLAS, SDPA, fused Adam, DDP/NCCL)"),
           "impl": "torch_eager_mx_linears" if args.mx else "torch_eager_baseline",
           "value": round(B * S * world / (ms / 1000.0), 1), "unit": "tokens/s",
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
           "dtype": "mxfp8 linears (E4M3 / E5M2, 1x32 UE8M0), bf16 elsewhere" if args.mx else "bf16 autocast", "data": "synthetic uniform-random tokens, N(0,0.02) init",
           "config": {"layers": args.layers, "d_model": d, "heads": h, "d_ff": f, "vocab": V, "seq_len": S,
                      "micro_batch_per_gpu": B, "params": nparams},
           "final_loss": round(float(loss), 4), "loss_is_finite": bool(math.isfinite(float(loss)))}
    if rank == 0:
        os.write(json_fd, (json.dumps(out) + "\n").encode())
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
