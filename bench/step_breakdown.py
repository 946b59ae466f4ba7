#!/usr/bin/env python
"""Where a GPT-1B training step spends its device time, kernel class by kernel class.

    python bench/step_breakdown.py [--precision fp8|mxfp8|bf16] [--steps 3] [--layers 24]

Runs the same step as ``bench.py`` (1 GPU, CUDA-graph replay), times ``--steps``
replays with CUDA events, then replays the same number of steps once more under
``torch.profiler`` (CUPTI kernel records: start / end of every kernel, no replay
of kernels, no serialisation) and sums the kernel durations per class.  The
table's rows are per step; ``busy`` is the union of all kernel intervals (so
kernels overlapping on two streams count once) and ``idle`` is the step time
minus ``busy``.  The CUDA-event step time, not the profiled one, is the step
time reported.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import sys
from collections import defaultdict

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

CLASSES = [  # (class, regex over the demangled kernel name); first match wins
    ("gemm fp8 (block GEMMs)", r"gemm_2sm_kernel<1"),
    ("gemm bf16 (LM head)", r"gemm_2sm_kernel<2|gemm_bf16_tn"),
    ("gemm mxfp8 plain (cuBLASLt)", r"bstensorop|block_scaled"),
    ("attention fwd", r"attn_fwd"),
    ("attention bwd", r"attn_bwd|attn_dq"),
    ("cross-entropy", r"xent"),
    ("adam / optimizer", r"adam|optim_finalize|grad_sumsq"),
    ("layernorm", r"ln_fwd|ln_bwd"),
    ("fp8 / mx quantise", r"quantize|mx_|amax|scaling_update"),
    ("bias-grad column sums", r"colsum"),
    ("embedding", r"embed"),
    ("nccl", r"nccl"),
    ("copies / fills", r"memcpy|memset|fill|copy|Memcpy|Memset"),
]


def classify(name: str) -> str:
    for cls, pat in CLASSES:
        if re.search(pat, name):
            return cls
    return "other"


def union_ms(intervals):
    tot, cur_s, cur_e = 0.0, None, None
    for s, e in sorted(intervals):
        if cur_e is None or s > cur_e:
            if cur_e is not None:
                tot += cur_e - cur_s
            cur_s, cur_e = s, e
        else:
            cur_e = max(cur_e, e)
    if cur_e is not None:
        tot += cur_e - cur_s
    return tot


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--precision", default="fp8", choices=["fp8", "mxfp8", "bf16"])
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--micro-batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--json", default=None, help="also write the table as JSON here")
    args = ap.parse_args()

    import torch
    from torch.profiler import ProfilerActivity, profile

    from mtorus.models.gpt import GptConfig
    from mtorus.training.engine import GptTrainer

    dev = torch.device("cuda", 0)
    cfg = GptConfig.gpt_1b_bench()
    if args.layers is not None:
        cfg.num_layers = args.layers
    B, S = args.micro_batch, args.seq
    tr = GptTrainer(cfg, device=dev, lr=3e-4, init="normal", seed=1234, fp8=args.precision != "bf16",
                    fp8_recipe="mx" if args.precision == "mxfp8" else "tensor")
    g = torch.Generator().manual_seed(7)
    t = torch.randint(0, cfg.vocab_size, (B, S + 1), generator=g)
    ids, tgt = t[:, :-1].contiguous().to(dev), t[:, 1:].contiguous().to(dev)
    for _ in range(args.warmup):
        tr.step_device(ids, tgt)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    tr.capture(ids, tgt)
    for _ in range(2):
        tr.graph_step(ids, tgt)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        tr.graph_step(ids, tgt)
    e1.record()
    e1.synchronize()
    step_ms = e0.elapsed_time(e1) / args.steps

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.steps):
            tr.graph_step(ids, tgt)
        torch.cuda.synchronize()
    per_cls = defaultdict(float)
    count = defaultdict(int)
    per_kernel = defaultdict(float)
    intervals = []
    gemm_seq = []  # (start, ms, name) of the block GEMM launches, in launch order
    t_lo, t_hi = None, None
    for ev in prof.events():
        if ev.device_type != torch.autograd.DeviceType.CUDA:
            continue
        dur_ms = ev.device_time / 1000.0 if hasattr(ev, "device_time") else ev.cuda_time / 1000.0
        if dur_ms <= 0:
            continue
        s = ev.time_range.start / 1000.0
        intervals.append((s, s + dur_ms))
        t_lo = s if t_lo is None else min(t_lo, s)
        t_hi = s + dur_ms if t_hi is None else max(t_hi, s + dur_ms)
        c = classify(ev.name)
        if c.startswith("gemm"):
            gemm_seq.append((s, dur_ms, c))
        per_cls[c] += dur_ms
        count[c] += 1
        per_kernel[ev.name] += dur_ms
    n = args.steps
    busy = union_ms(intervals) / n
    span = (t_hi - t_lo) / n if intervals else 0.0
    rows = sorted(((c, v / n, count[c] / n) for c, v in per_cls.items()), key=lambda r: -r[1])
    total = sum(r[1] for r in rows)
    out = {"precision": args.precision, "layers": cfg.num_layers, "tokens_per_step": B * S,
           "step_ms_cuda_events": round(step_ms, 3), "profiled_span_ms": round(span, 3),
           "kernel_sum_ms": round(total, 3), "busy_union_ms": round(busy, 3),
           "idle_ms": round(max(0.0, step_ms - busy), 3),
           "rows": [{"class": c, "ms_per_step": round(v, 3), "launches_per_step": round(k, 1),
                     "share_of_step": round(v / step_ms, 4)} for c, v, k in rows],
           "top_kernels": [{"name": k[:160], "ms_per_step": round(v / n, 3)}
                           for k, v in sorted(per_kernel.items(), key=lambda kv: -kv[1])[:25]]}
    print(f"step {step_ms:.3f} ms (CUDA events, {n} graph replays); profiled span {span:.3f} ms; "
          f"kernel sum {total:.3f} ms; busy (union) {busy:.3f} ms; idle {max(0.0, step_ms - busy):.3f} ms")
    print(f"{'class':32s} {'ms/step':>9s} {'share':>7s} {'launches':>9s}")
    for c, v, k in rows:
        print(f"{c:32s} {v:9.3f} {v / step_ms:7.1%} {k:9.1f}")
    gemm_seq.sort()
    fp8 = [d for _, d, c in gemm_seq if c.startswith("gemm fp8") or c.startswith("gemm mxfp8")]
    per_step = len(fp8) // n if n else 0
    if per_step >= 24:
        first = fp8[:per_step]
        bwd = first[per_step - 8:]
        out["layer0_fwd_gemm_ms"] = [round(x, 4) for x in first[4:8]]
        out["layer0_bwd_gemm_ms"] = [round(x, 4) for x in bwd]
        print("one layer's forward GEMMs (qkv, out, ffn1, ffn2), ms:", out["layer0_fwd_gemm_ms"])
        print("layer 0 backward GEMMs in launch order, ms:", out["layer0_bwd_gemm_ms"])
    print("top kernels:")
    for r in out["top_kernels"]:
        print(f"  {r['ms_per_step']:8.3f}  {r['name']}")
    if args.json:
        with open(args.json, "w") as f:
            json.dump(out, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
