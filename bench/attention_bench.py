#!/usr/bin/env python
"""Causal attention forward / backward timing: the tcgen05 kernels of
``csrc/kernels/attention.cu`` vs torch's scaled_dot_product_attention (whatever
backend torch selects: cuDNN or flash) on the GPT-1B shape.

    python bench/attention_bench.py --batch 8 --seq 2048 --heads 16

One JSON line per (impl, pass) with ms and TFLOP/s (causal: half the S^2 work;
backward counted as 2.5x forward).  CUDA-event timing after warm-up; inputs
(qkv 8 x 2048 x 6144 bf16 = 201 MB) exceed L2.
"""
import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402


def timeit(fn, iters, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) / iters


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args()
    from mtorus.ops.attention import attention_bwd, attention_fwd

    B, S, H, dh = args.batch, args.seq, args.heads, 128
    torch.manual_seed(0)
    qkv = torch.randn(B * S, 3 * H * dh, device="cuda").bfloat16()
    dout = torch.randn(B * S, H * dh, device="cuda").bfloat16()
    fl_fwd = 4.0 * B * H * S * S * dh / 2
    out, lse = attention_fwd(qkv, B, S, H)
    rows = []
    t = timeit(lambda: attention_fwd(qkv, B, S, H), args.iters)
    rows.append(("mtorus", "fwd", t, fl_fwd))
    t = timeit(lambda: attention_bwd(dout, qkv, out, lse, B, S, H), args.iters)
    rows.append(("mtorus", "bwd", t, 2.5 * fl_fwd))

    q, k, v = (x.transpose(1, 2) for x in qkv.view(B, S, 3, H, dh).unbind(2))
    q, k, v = (x.detach().requires_grad_(True) for x in (q, k, v))
    t = timeit(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True), args.iters)
    rows.append(("torch_sdpa", "fwd", t, fl_fwd))
    o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    g = torch.randn_like(o)
    t = timeit(lambda: torch.autograd.grad(o, (q, k, v), g, retain_graph=True), args.iters)
    rows.append(("torch_sdpa", "bwd", t, 2.5 * fl_fwd))
    for impl, p, ms, fl in rows:
        print(json.dumps({"impl": impl, "pass": p, "B": B, "S": S, "H": H, "dh": dh, "ms": round(ms, 4),
                          "tflops": round(fl / ms / 1e9, 1)}), flush=True)


if __name__ == "__main__":
    main()
