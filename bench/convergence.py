#!/usr/bin/env python
"""Loss curves of one GPT configuration under several GEMM precisions, on data a
model can learn: the same seed, the same weights and the same token stream for
every precision, so the curves differ only by the GEMM arithmetic.

    python bench/convergence.py --steps 60 --precisions bf16,fp8,mxfp8,mxfp8/head-bf16

Data: a fixed random first-order Markov chain over the first ``--active-vocab``
token ids (of the model's full vocabulary) in which every token has ``--branching``
equally likely successors, so the achievable loss is ln(branching) (1.39 nats for 4)
while a fresh model starts near ln(V): within a few steps it learns which ids occur
(ln(active-vocab)), then the transitions.  Each step
draws a new batch from the chain (host RNG, seeded), copies it in, and runs one
``GptTrainer.step_device``.  A precision with the suffix ``/head-bf16`` keeps the LM
head in bf16 (the FP8 precisions run it in FP8 by default).  Prints one JSON line per
precision with the loss every
step, then one summary line: the largest absolute gap of each precision's loss to
the bf16 curve over the last quarter of the steps.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def markov_batches(vocab: int, branching: int, batch: int, seq: int, steps: int, seed: int):
    """steps batches of [batch, seq + 1] tokens in [0, vocab) from a fixed random Markov chain."""
    import torch

    g = torch.Generator().manual_seed(seed)
    succ = torch.randint(0, vocab, (vocab, branching), generator=g)
    n = steps * batch
    t = torch.empty(n, seq + 1, dtype=torch.long)
    t[:, 0] = torch.randint(0, vocab, (n,), generator=g)
    pick = torch.randint(0, branching, (n, seq), generator=g)
    for s in range(seq):  # the chain is sequential along s; rows advance together
        t[:, s + 1] = succ[t[:, s], pick[:, s]]
    return list(t.split(batch))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--precisions", default="bf16,fp8,mxfp8,mxfp8/head-bf16")
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--micro-batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--branching", type=int, default=4)
    ap.add_argument("--active-vocab", type=int, default=1024, help="token ids the chain uses (<= the vocabulary)")
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--warmup", type=int, default=10, help="linear learning-rate warmup steps")
    ap.add_argument("--seed", type=int, default=1234)
    args = ap.parse_args(argv)

    import torch

    from mtorus.models.gpt import GptConfig
    from mtorus.training.engine import GptTrainer

    cfg = GptConfig.gpt_1b_bench()
    cfg.num_layers = args.layers
    batches = markov_batches(min(args.active_vocab, cfg.vocab_size), args.branching, args.micro_batch, args.seq,
                             args.steps, args.seed)
    curves = {}
    for prec in args.precisions.split(","):
        base_prec, _, opt = prec.partition("/")
        tr = GptTrainer(cfg, device="cuda", lr=args.lr, init="normal", seed=args.seed, dp="none",
                        warmup_steps=args.warmup, fp8=base_prec in ("fp8", "mxfp8"),
                        fp8_recipe="mx" if base_prec == "mxfp8" else "tensor", fp8_head=opt != "head-bf16")
        losses = []
        for t in batches:
            ids = t[:, :-1].contiguous().cuda(non_blocking=True)
            tgt = t[:, 1:].contiguous().cuda(non_blocking=True)
            losses.append(float(tr.step_device(ids, tgt)))
        curves[prec] = losses
        print(json.dumps({"precision": prec, "steps": args.steps, "losses": [round(x, 5) for x in losses]}),
              flush=True)
        del tr
        torch.cuda.empty_cache()
    base = curves.get("bf16")
    tail = max(1, args.steps // 4)
    summary = {"model": f"GPT-1B shape, {cfg.num_layers} layers", "tokens_per_step": args.micro_batch * args.seq,
               "data": f"random Markov chain over {min(args.active_vocab, cfg.vocab_size)} token ids, "
                       f"{args.branching} successors per token (floor ln {args.branching} = "
                       f"{torch.log(torch.tensor(float(args.branching))).item():.3f})",
               "final_loss": {p: round(c[-1], 4) for p, c in curves.items()}}
    if base is not None:
        summary["max_abs_gap_to_bf16_last_quarter"] = {
            p: round(max(abs(a - b) for a, b in zip(c[-tail:], base[-tail:])), 4) for p, c in curves.items()
            if p != "bf16"}
    print(json.dumps(summary), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
