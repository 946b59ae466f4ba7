#!/usr/bin/env python
"""Train a GPT on B200 GPUs with the fused sm_100a path.

    # one GPU, GPT-1B, FP8, 20 steps, metrics as JSON lines
    python examples/gpt1b/train_gpu.py --model gpt1b --steps 20 --metrics run.jsonl
    # 8 GPUs: data parallel over the NVLink-fused reducer, checkpoints every 100 steps
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/gpt1b/train_gpu.py \\
        --config train.toml --set learning_rate=3e-4 --set checkpoint_interval=100 \\
        --dp symm --checkpoint-dir ckpt
    # 8 GPUs: DP 2 x PP 4 with the 1F1B schedule from the config
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/gpt1b/train_gpu.py \\
        --set 'pipeline_schedule={OneF1B={num_stages=4}}' --set accumulation_steps=16

The TrainingConfig (TOML file and ``--set key=value`` overrides, values in TOML
syntax) supplies: learning_rate, warmup_steps, clip_grad_norm, micro_batch_size
(sequences per GPU per micro-batch), accumulation_steps (micro-batches per
optimizer step; the pipeline's micro-batch count when pipelined),
pipeline_schedule (GPipe / OneF1B{num_stages}: pipeline parallel over
num_stages GPUs, the rest data parallel), mixed_precision.scaling_strategy
(Dynamic -> dynamic loss scaling from 2^16; Delayed{history_length} -> FP8 amax
history length), checkpoint_interval and log_interval (the reference's
TrainingConfig, crates/mt-training/src/config.rs).  Data: synthetic uniform
tokens (next-token targets) from a seed.  ``--resume DIR`` continues from a
checkpoint (restored exactly).
"""
from __future__ import annotations

import argparse
import os
import sys
from datetime import timedelta

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))


def parse_set(items, base: dict) -> dict:
    """Apply ``key=value`` overrides (dotted keys into nested tables, TOML values)."""
    import tomllib

    for it in items or []:
        key, _, val = it.partition("=")
        try:
            v = tomllib.loads(f"v = {val}")["v"]
        except Exception:
            v = val
        d = base
        parts = key.strip().split(".")
        for p in parts[:-1]:
            d = d.setdefault(p, {})
        d[parts[-1]] = v
    return base


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default=None, help="TrainingConfig TOML file")
    ap.add_argument("--set", action="append", default=[], help="override: key=value (TOML value)")
    ap.add_argument("--model", default="gpt1b", choices=["gpt1b", "gpt6.7b", "small"])
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--dp", default="nccl", choices=["nccl", "symm"])
    ap.add_argument("--bf16", action="store_true", help="bf16 block GEMMs instead of FP8")
    ap.add_argument("--numa-bind", action="store_true",
                    help="pin each rank's host threads to the CPUs of its GPU's NUMA node")
    ap.add_argument("--fp8-recipe", default="tensor", choices=["tensor", "mx"],
                    help="tensor: per-tensor delayed scaling; mx: MXFP8 1x32 block scales in all block GEMMs")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--metrics", default=None, help="append per-step JSON lines here (rank 0)")
    ap.add_argument("--checkpoint-dir", default=None)
    ap.add_argument("--resume", default=None)
    args = ap.parse_args(argv)

    import torch
    import torch.distributed as dist

    from mtorus.core.precision import ScalingStrategy
    from mtorus.models.gpt import GptConfig
    from mtorus.training.checkpoint import load_checkpoint, maybe_save
    from mtorus.training.config import PipelineScheduleConfig, TrainingConfig
    from mtorus.training.fused_optim import DeviceLossScaleConfig
    from mtorus.utils.metrics import MetricsLogger

    base = TrainingConfig.load(args.config).to_dict() if args.config else TrainingConfig(
        batch_size=8, micro_batch_size=8, accumulation_steps=1, learning_rate=3e-4).to_dict()
    tc = TrainingConfig.from_dict(parse_set(args.set, base))
    tc.validate()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.numa_bind:
        from mtorus.core.topology import bind_to_gpu_numa

        bind_to_gpu_numa(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    cfg = {"gpt1b": GptConfig.gpt_1b_bench(), "gpt6.7b": GptConfig.gpt_6_7b(),
           "small": GptConfig(vocab_size=4096, d_model=512, num_layers=4, num_heads=4, d_ff=2048,
                              max_seq_len=args.seq, dropout=0.0)}[args.model]
    S = args.seq
    mp = tc.mixed_precision
    dynamic = isinstance(mp.scaling_strategy, ScalingStrategy.Dynamic)
    history = 16 if dynamic else int(mp.scaling_strategy.history_length)
    ls = DeviceLossScaleConfig(init_scale=65536.0 if dynamic else 1.0, dynamic=dynamic, growth_interval=2000)
    b, M = tc.micro_batch_size, tc.accumulation_steps
    pp = tc.pipeline_schedule.num_stages if isinstance(tc.pipeline_schedule, PipelineScheduleConfig.OneF1B) else 1
    if pp > 1:
        from mtorus.pipeline.schedule import ScheduleType
        from mtorus.training.pipeline_engine import PipelineTrainer

        if world % pp:
            raise SystemExit(f"world size {world} is not a multiple of num_stages {pp}")
        tr = PipelineTrainer(cfg, pp=pp, dp=world // pp, schedule=ScheduleType.OneF1B, num_microbatches=M,
                             micro_batch=b, seq_len=S, fp8=not args.bf16, fp8_history=history,
                             fp8_recipe=args.fp8_recipe, lr=tc.learning_rate, device=dev, seed=args.seed,
                             loss_scale=ls, max_grad_norm=tc.clip_grad_norm)
        replicas = world // pp
        replica = tr.replica
    else:
        from mtorus.training.engine import GptTrainer

        tr = GptTrainer(cfg, device=dev, lr=tc.learning_rate, init="normal", seed=args.seed, dp=args.dp,
                        loss_scale=ls, max_grad_norm=tc.clip_grad_norm, warmup_steps=tc.warmup_steps,
                        fp8=not args.bf16, fp8_history=history, fp8_recipe=args.fp8_recipe)
        replicas, replica = world, rank
    if args.resume:
        load_checkpoint(args.resume, tr)

    gen = torch.Generator().manual_seed(args.seed * 7919 + replica)
    log = MetricsLogger(args.metrics if rank == 0 else None, tokens_per_step=replicas * M * b * S)
    for _ in range(args.steps):
        t = torch.randint(0, cfg.vocab_size, (M, b, S + 1), generator=gen)
        ids, tgt = t[..., :-1].contiguous().pin_memory(), t[..., 1:].contiguous().pin_memory()
        if pp > 1:
            loss = tr.train_step(ids if tr.is_first else None, tgt if tr.is_last else None)
            lt = torch.tensor([loss if loss is not None else 0.0], device=dev)
            dist.broadcast(lt, tr.layout.stage_ranks[0][-1])
            loss = float(lt)
        else:
            d_ids = [x.to(dev, non_blocking=True) for x in ids.unbind(0)]
            d_tgt = [x.to(dev, non_blocking=True) for x in tgt.unbind(0)]
            loss = float(tr.step_device_accum(d_ids, d_tgt))
        st = tr.opt.stats()
        log.log(tr.global_step, loss, tc.learning_rate, st["grad_norm"], st["skipped"], st["loss_scale"])
        if rank == 0 and tc.log_interval and tr.global_step % tc.log_interval == 0:
            print(f"Step {tr.global_step:3} | loss = {loss:.6f}", flush=True)
        if args.checkpoint_dir:
            maybe_save(args.checkpoint_dir, tr, tc)
    if rank == 0:
        print(log.summary(), flush=True)
    log.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
