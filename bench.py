#!/usr/bin/env python
"""GPT-1B training throughput benchmark (tokens/s, device-timed, max over ranks).

Workload: GPT-1B decoder (24 layers, d_model 2048, 16 heads, d_ff 8192, vocab
50304, seq 2048), micro-batch 8 sequences per GPU, pure data parallel over
NCCL process groups, uniform-random synthetic tokens, N(0, 0.02) random-init
weights, Adam.  One step = forward + backward + gradient reduction + optimizer.
The transformer-layer GEMMs run the FP8 recipe with 1x32 block scales (MXFP8:
E4M3 forward, E5M2 gradients, one UE8M0 scale per 32 values) unless
``--precision`` says otherwise.

    python bench.py --gpus 1 --steps 10 --warmup 3
    torchrun --nproc-per-node 8 bench.py --gpus 8 ...

Rank 0 prints one JSON line.  ``value`` is the whole-job tokens/s over all GPUs
(weak scaling: per-GPU work fixed).  ``e2e`` repeats the measurement through
the public ``GptTrainer.train_step`` API with pinned host batches copied in and
the loss read back every step.

``--impl reference`` reports why the reference implementation cannot run here.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from datetime import timedelta

REF_UNAVAILABLE = ("reference is a Rust/Burn CPU crate workspace with no Python package, no GPU or "
                   "NCCL path and no Rust toolchain on this machine; pip install of it fails "
                   "(neither setup.py nor pyproject.toml)")


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def _mx_library() -> bool:
    from mtorus.ops import mxfp8

    return mxfp8.LIBRARY_PLAIN_GEMM


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mtorus", choices=["mtorus", "reference"])
    ap.add_argument("--micro-batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--dp", default="symm", choices=["nccl", "symm"],
                    help="symm (default): fused NVLink reduce-scatter + sharded Adam + weight all-gather over "
                         "symmetric memory; nccl: NCCL bucket all-reduce + full Adam on every rank (the baseline)")
    ap.add_argument("--layers", type=int, default=None,
                    help="override layer count (debug only; the metric is defined for 24)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--graph", default="auto", choices=["auto", "on", "off"],
                    help="replay the whole step as one CUDA graph (any --dp); auto: on")
    ap.add_argument("--lm-head", default="fp8", choices=["fp8", "bf16"],
                    help="LM-head GEMMs in FP8 (per-tensor delayed scaling, E4M3 / E5M2) or bf16 "
                         "(ignored with --precision bf16)")
    ap.add_argument("--precision", default="mxfp8", choices=["mxfp8", "fp8", "bf16"],
                    help="mxfp8 (default): E4M3 / E5M2 with one UE8M0 scale per 1x32 block in every "
                         "transformer-layer GEMM (block-scaled tcgen05 GEMMs); fp8: the same formats with one "
                         "per-tensor delayed-scaling scale; bf16: all GEMMs bf16")
    args = ap.parse_args()

    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": REF_UNAVAILABLE}))
        return 0

    # Libraries (NCCL's version banner, extension builds) may write to stdout; the
    # contract is one JSON line there, so fd 1 goes to stderr until the result is out.
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)

    import torch
    import torch.distributed as dist

    from mtorus._ext import cuda as _cuda
    from mtorus.models.gpt import GptConfig
    from mtorus.training.engine import GptTrainer
    from mtorus.utils.clocks import ClockSampler

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        log(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    cfg = GptConfig.gpt_1b_bench()
    if args.layers is not None:
        cfg.num_layers = args.layers
    B, S = args.micro_batch, args.seq
    trainer = GptTrainer(cfg, device=dev, lr=3e-4, init="normal", seed=1234, dp=args.dp,
                         fp8=args.precision in ("fp8", "mxfp8"),
                         fp8_recipe="mx" if args.precision == "mxfp8" else "tensor",
                         fp8_head=args.lm_head == "fp8")
    ext = _cuda()

    # synthetic next-token data: uniform ids, targets shifted by one
    nb = 4
    gen = torch.Generator().manual_seed(1000 + rank)
    host_ids, host_tgt = [], []
    for _ in range(nb):
        t = torch.randint(0, cfg.vocab_size, (B, S + 1), generator=gen)
        host_ids.append(t[:, :-1].contiguous().pin_memory())
        host_tgt.append(t[:, 1:].contiguous().pin_memory())
    dev_ids = [x.to(dev) for x in host_ids]
    dev_tgt = [x.to(dev) for x in host_tgt]

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for i in range(args.warmup):
        trainer.step_device(dev_ids[i % nb], dev_tgt[i % nb])
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    use_graph = args.graph in ("on", "auto")
    if use_graph:
        torch.cuda.empty_cache()
        trainer.capture(dev_ids[0], dev_tgt[0])
        for i in range(2):  # the replays' own warm-up
            trainer.graph_step(dev_ids[i % nb], dev_tgt[i % nb])
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
    step_fn = trainer.graph_step if use_graph else trainer.step_device

    sampler = ClockSampler(local_rank).start()
    time.sleep(0.3)
    lc0 = ext.launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    h0 = time.perf_counter()
    for i in range(args.steps):
        loss = step_fn(dev_ids[i % nb], dev_tgt[i % nb])
    host_ms = (time.perf_counter() - h0) * 1000.0
    t1.record()
    t1.synchronize()
    lc1 = ext.launch_count()
    if use_graph:  # graph replays launch the captured kernels without host launches
        lc1 += trainer.graph_launches * args.steps
    barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = t0.elapsed_time(t1)
    last_loss = float(loss)

    # exposed communication: the same steps with no data-parallel traffic at all
    comp_ms = None
    if world > 1:
        barrier()
        torch.cuda.synchronize()
        for i in range(2):
            trainer.step_device(dev_ids[i % nb], dev_tgt[i % nb], reduce=False)
        comp_fn = lambda a, b: trainer.step_device(a, b, reduce=False)  # noqa: E731
        if use_graph:
            trainer.capture(dev_ids[0], dev_tgt[0], reduce=False)
            trainer.graph_step(dev_ids[0], dev_tgt[0], reduce=False)
            comp_fn = lambda a, b: trainer.graph_step(a, b, reduce=False)  # noqa: E731
        torch.cuda.synchronize()
        barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record()
        for i in range(args.steps):
            comp_fn(dev_ids[i % nb], dev_tgt[i % nb])
        c1.record()
        c1.synchronize()
        comp_ms = c0.elapsed_time(c1)
        barrier()

    e2e_ms = None
    if not args.no_e2e:
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            trainer.train_step(host_ids[i % nb], host_tgt[i % nb])
        e1.record()
        e1.synchronize()
        e2e_ms = e0.elapsed_time(e1)
        barrier()

    if world > 1:
        t = torch.tensor([ms, e2e_ms or 0.0, comp_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, comp_ms = float(t[0]), (float(t[1]) if e2e_ms is not None else None), float(t[2])

    tokens_per_step = B * S * world
    ms_step = ms / args.steps
    value = tokens_per_step / (ms_step / 1000.0)
    head = ("LM-head GEMMs FP8 (E4M3 h / weight, E5M2 dlogits, per-tensor delayed scaling)"
            if args.lm_head == "fp8" else "bf16 LM head")
    out = {
        "metric": "GPT-1B FP8 tokens/sec (device-timed, max over ranks) at 1/2/4/8 B200; exposed comm/step",
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": {"fp8": "fp8 (transformer-layer GEMMs: E4M3 forward / E5M2 gradients, one per-tensor "
                         "delayed-scaling scale per operand; " + head + "; bf16 attention, activations; fp32 "
                         "master weights / Adam)",
                  "mxfp8": "mxfp8 (transformer-layer GEMMs: E4M3 forward / E5M2 gradients, one UE8M0 scale per "
                           "1x32 block along each GEMM's contraction dimension; " + head + "; bf16 attention, "
                           "activations; fp32 master weights / Adam)",
                  "bf16": "bf16"}[args.precision],
        "data": "synthetic uniform-random tokens, random-init N(0,0.02) weights",
        "config": {
            "lm_head": args.lm_head if args.precision != "bf16" else "bf16",
            "model": f"GPT-1B ({cfg.num_layers} layers, d_model {cfg.d_model}, {cfg.num_heads} heads, "
                     f"d_ff {cfg.d_ff}, vocab {cfg.vocab_size})",
            "global_batch": B * world,
            "seq_len": S,
            "micro_batch_per_gpu": B,
            "parallelism": f"dp{world}",
            "dp_reduce": args.dp if world > 1 else "none",
            "dp_grad_transport": ("e5m2 (1x32 power-of-two scales)" if os.environ.get("MTORUS_DP_GRAD_FP8") == "1"
                                  else "fp32") if world > 1 else "none",
            "precision": args.precision,
            "gemm": {"fp8": "tcgen05 kind::f8f6f4 fp8 + kind::f16 bf16, CTA-pair 256x256 tiles, fp32 accumulate",
                     "mxfp8": "tcgen05 kind::mxf8f6f4 block-scaled fp8 + kind::f16 bf16, CTA-pair 256x256 tiles, "
                              "fp32 accumulate" + ("; plain GEMMs (bias-only epilogue, fresh output) on cuBLASLt MXFP8"
                                                   if _mx_library() else ""),
                     "bf16": "tcgen05 kind::f16 bf16, CTA-pair 256x256 tiles"}[args.precision],
            "l2": "per-step working set (activations, 1.4B-param optimizer state) >> 126 MB L2; no flush",
            "params": cfg.num_params(),
            "model_tflops_per_gpu": round(cfg.train_flops_per_token(S) * B * S / (ms_step / 1000.0) / 1e12, 1),
        },
        "exposed_comm": {
            "ms_per_step": round(max(0.0, ms_step - comp_ms / args.steps), 3) if comp_ms is not None else 0.0,
            "fraction_of_step": (round(max(0.0, ms_step - comp_ms / args.steps) / ms_step, 4)
                                 if comp_ms is not None else 0.0),
            "compute_only_ms_per_step": round(comp_ms / args.steps, 3) if comp_ms is not None else round(ms_step, 3),
            "how": "device-timed step minus the same step with no data-parallel communication (max over ranks)",
        },
        "host_enqueue_ms_per_step": round(host_ms / args.steps, 3),
        "cuda_graph": use_graph,
        "clocks": clocks,
        "gpu_launches": int(lc1 - lc0),
        "final_loss": round(last_loss, 4),
    }
    if e2e_ms is not None:
        out["e2e"] = {
            "value": round(tokens_per_step / (e2e_ms / args.steps / 1000.0), 1),
            "unit": "tokens/s",
            "h2d_bytes_per_step": int(host_ids[0].numel() * host_ids[0].element_size()
                                      + host_tgt[0].numel() * host_tgt[0].element_size()),
            "d2h_bytes_per_step": 4,
            "api": "mtorus.training.engine.GptTrainer.train_step",
        }
    if rank == 0:
        os.write(json_fd, (json.dumps(out) + "\n").encode())
    trainer.release_graphs()  # a graph holding NCCL calls must go before the process group
    if world > 1:
        barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
