#!/usr/bin/env python
"""GPT training throughput with data x pipeline parallelism (NCCL p2p stages).

    torchrun --nproc-per-node 8 bench/gpt_pipeline.py --model gpt1b --dp 2 --pp 4 \\
        --schedule 1f1b --micro-batches 16 --micro-batch 4
    torchrun --nproc-per-node 8 bench/gpt_pipeline.py --model gpt6.7b --dp 1 --pp 8 \\
        --schedule gpipe --micro-batches 32 --micro-batch 2

Synthetic uniform-random tokens, N(0, 0.02) random-init weights, FP8 block GEMMs
(E4M3 forward / E5M2 gradients, delayed scaling), full activation checkpointing
per stage (``--no-checkpoint`` to keep activations).  Every step: M micro-batches
through the schedule, data-parallel gradient all-reduce (dp > 1), Adam.

Rank 0 prints one JSON line: whole-job tokens/s (device-timed, max over ranks),
the measured pipeline bubble (idle share of each rank's compute span, averaged
and max over ranks) next to the schedule's ideal (S-1)/(M+S-1), and an
end-to-end number through ``PipelineTrainer.train_step`` (pinned host batches
copied in, loss read back every step).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from datetime import timedelta

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def main(argv=None, defaults=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="gpt1b", choices=["gpt1b", "gpt6.7b"])
    ap.add_argument("--dp", type=int, default=2)
    ap.add_argument("--pp", type=int, default=4)
    ap.add_argument("--schedule", default="1f1b", choices=["1f1b", "gpipe"])
    ap.add_argument("--micro-batches", type=int, default=16)
    ap.add_argument("--micro-batch", type=int, default=4)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--no-checkpoint", action="store_true")
    ap.add_argument("--precision", default="fp8", choices=["fp8", "mxfp8", "bf16"])
    ap.add_argument("--lm-head", default="fp8", choices=["fp8", "bf16"],
                    help="LM-head GEMMs in FP8 (per-tensor delayed scaling) or bf16")
    ap.add_argument("--dp-mode", default="symm", choices=["symm", "nccl"],
                    help="symm: fused NVLink reduce-scatter + sharded Adam + amax all-reduce in the quantise "
                         "kernels; nccl: NCCL bucket all-reduce (the baseline)")
    ap.add_argument("--checkpoint", default="full", choices=["full", "selective", "none"])
    ap.add_argument("--wire", default="native", choices=["native", "fp8"],
                    help="stage transfers as bf16 or as block-scaled FP8 codes")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--layers", type=int, default=None, help="override layer count (debug only)")
    if defaults:
        ap.set_defaults(**defaults)
    args = ap.parse_args(argv)

    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)
    if os.environ.get("MTORUS_HANG_DUMP"):
        import faulthandler

        faulthandler.dump_traceback_later(int(os.environ["MTORUS_HANG_DUMP"]), exit=False)

    import torch
    import torch.distributed as dist

    from mtorus._ext import cuda as _cuda
    from mtorus.models.gpt import GptConfig
    from mtorus.pipeline.checkpoint import CheckpointStrategy
    from mtorus.pipeline.schedule import ScheduleType
    from mtorus.training.pipeline_engine import PipelineTrainer
    from mtorus.utils.clocks import ClockSampler

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    if world != args.dp * args.pp:
        raise SystemExit(f"WORLD_SIZE {world} != dp {args.dp} x pp {args.pp}")

    cfg = GptConfig.gpt_1b_bench() if args.model == "gpt1b" else GptConfig.gpt_6_7b()
    if args.layers is not None:
        cfg.num_layers = args.layers
    sched = ScheduleType.OneF1B if args.schedule == "1f1b" else ScheduleType.Gpipe
    ckpt = {"full": CheckpointStrategy.Full, "selective": CheckpointStrategy.Selective,
            "none": CheckpointStrategy.None_}["none" if args.no_checkpoint else args.checkpoint]
    M, b, S = args.micro_batches, args.micro_batch, args.seq
    tr = PipelineTrainer(cfg, pp=args.pp, dp=args.dp, schedule=sched, num_microbatches=M, micro_batch=b,
                         seq_len=S, checkpoint=ckpt, fp8=args.precision in ("fp8", "mxfp8"), lr=3e-4, device=dev,
                         seed=1234, fp8_recipe="mx" if args.precision == "mxfp8" else "tensor",
                         fp8_head=args.lm_head == "fp8",
                         dp_mode=args.dp_mode if args.dp > 1 else "nccl", wire=args.wire)
    ext = _cuda()

    gen = torch.Generator().manual_seed(1000 + tr.replica)
    nb = 2
    host_ids, host_tgt = [], []
    for _ in range(nb):
        t = torch.randint(0, cfg.vocab_size, (M, b, S + 1), generator=gen)
        host_ids.append(t[:, :, :-1].contiguous().pin_memory())
        host_tgt.append(t[:, :, 1:].contiguous().pin_memory())
    dev_ids = [list(x.to(dev).unbind(0)) for x in host_ids]
    dev_tgt = [list(x.to(dev).unbind(0)) for x in host_tgt]

    def barrier():
        dist.barrier(device_ids=[local_rank])

    for i in range(args.warmup):
        tr.step_device(dev_ids[i % nb], dev_tgt[i % nb])
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()

    sampler = ClockSampler(local_rank).start()
    time.sleep(0.3)
    lc0 = ext.launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    loss = None
    for i in range(args.steps):
        loss = tr.step_device(dev_ids[i % nb], dev_tgt[i % nb])
    t1.record()
    t1.synchronize()
    lc1 = ext.launch_count()
    barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = t0.elapsed_time(t1)

    # bubble: one more step with events around every forward / backward
    tr.executor.timed = True
    tr.step_device(dev_ids[0], dev_tgt[0])
    torch.cuda.synchronize()
    tr.executor.timed = False
    bubble = torch.tensor([tr.executor.bubble_fraction or 0.0], device=dev)
    bub_all = [torch.zeros_like(bubble) for _ in range(world)]
    dist.all_gather(bub_all, bubble)
    bubbles = [float(x) for x in bub_all]

    e2e_ms = None
    if not args.no_e2e:
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            tr.train_step(host_ids[i % nb] if tr.is_first else None, host_tgt[i % nb] if tr.is_last else None)
        e1.record()
        e1.synchronize()
        e2e_ms = e0.elapsed_time(e1)
        barrier()

    t = torch.tensor([ms, e2e_ms or 0.0], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = float(t[0]), (float(t[1]) if e2e_ms is not None else None)
    # the loss lives on the last stage of replica 0
    last_rank = tr.layout.stage_ranks[0][-1]
    lt = torch.zeros(1, device=dev)
    if rank == last_rank and loss is not None:
        lt.copy_(loss.reshape(1))
    dist.broadcast(lt, last_rank)

    tokens_per_step = args.dp * M * b * S
    ms_step = ms / args.steps
    value = tokens_per_step / (ms_step / 1000.0)
    name = "GPT-1B" if args.model == "gpt1b" else "GPT-6.7B"
    out = {
        "metric": f"{name} FP8 DP{args.dp}xPP{args.pp} {args.schedule} training tokens/sec (device-timed, max over ranks)",
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": {"fp8": "fp8 (transformer-layer GEMMs: E4M3 forward / E5M2 gradients, per-tensor delayed "
                         "scaling; LM head " + args.lm_head + "; bf16 attention, activations; fp32 master weights / Adam)",
                  "mxfp8": "mxfp8 (transformer-layer GEMMs: E4M3 forward / E5M2 gradients, one UE8M0 scale per "
                           "1x32 block; LM head " + args.lm_head + " (per-tensor); bf16 attention, activations; "
                           "fp32 master weights / Adam)",
                  "bf16": "bf16"}[args.precision],
        "data": "synthetic uniform-random tokens, random-init N(0,0.02) weights",
        "config": {
            "model": f"{name} ({cfg.num_layers} layers, d_model {cfg.d_model}, {cfg.num_heads} heads, "
                     f"d_ff {cfg.d_ff}, vocab {cfg.vocab_size})",
            "global_batch": args.dp * M * b,
            "seq_len": S,
            "micro_batches": M,
            "micro_batch": b,
            "parallelism": f"dp{args.dp}xpp{args.pp}",
            "schedule": args.schedule,
            "activation_checkpointing": "none" if args.no_checkpoint else f"{args.checkpoint} per stage",
            "dp_reduce": (args.dp_mode if args.dp > 1 else "none"),
            "stage_transfer": ("NCCL p2p, " + ("block-scaled FP8 (E4M3 activations / E5M2 gradients)"
                                               if args.wire == "fp8" else "bf16 activations / gradients")
                               + ", separate groups per direction"),
            "l2": "per-step working set >> 126 MB L2; no flush",
            "model_tflops_per_gpu": round(cfg.train_flops_per_token(S) * tokens_per_step / world
                                          / (ms_step / 1000.0) / 1e12, 1),
        },
        "bubble_fraction": {"measured_mean": round(sum(bubbles) / len(bubbles), 4),
                            "measured_max": round(max(bubbles), 4),
                            "ideal": round(tr.ideal_bubble_fraction(), 4),
                            "per_rank": [round(x, 4) for x in bubbles]},
        "clocks": clocks,
        "gpu_launches": int(lc1 - lc0),
        "final_loss": round(float(lt), 4),
    }
    if e2e_ms is not None:
        out["e2e"] = {
            "value": round(tokens_per_step / (e2e_ms / args.steps / 1000.0), 1),
            "unit": "tokens/s",
            # per replica: token ids into the first stage, targets into the last
            "h2d_bytes_per_step": int(host_ids[0].numel() * host_ids[0].element_size()
                                      + host_tgt[0].numel() * host_tgt[0].element_size()),
            "d2h_bytes_per_step": 4,
            "api": "mtorus.training.pipeline_engine.PipelineTrainer.train_step",
        }
    if rank == 0:
        os.write(json_fd, (json.dumps(out) + "\n").encode())
    barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
