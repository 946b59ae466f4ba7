#!/usr/bin/env python
"""GPT example on the CPU: data x pipeline parallelism in one process.

The reference's gpt-1b example (examples/gpt-1b/src/main.rs:43-115) builds a
tiny GPT, a one-rank MockCommunicator and a DistributedRuntime, then trains
with plain Adam; FP8, the pipeline and the communicator are never exercised.
This example runs the same model with all of them:

* model: GPT decoder, 2 layers, d_model 128, 4 heads, d_ff 512, vocab 1024,
  seq 64, dropout 0.1 (``GptConfig.example_tiny``), uniform-random tokens from a
  seed, next-token cross-entropy;
* world: 4 ranks of a single-process ``MockCommunicator`` world laid on a 2x2
  ``MeshTorusHybrid`` (one device per node): 2 data-parallel replicas x 2
  pipeline stages, stage ranks from ``topology_aware_placement``;
* pipeline: 1F1B over the 2 stages with 4 micro-batches per step (op lists from
  the schedule builder), stage transfers as FP8 frames through ``PipelineComm``
  (activations E4M3, gradients E5M2);
* precision: every Linear in FP8 with delayed scaling (E4M3 forward, E5M2
  backward, amax history 16), dynamic loss scaling from 2^16;
* data parallel: after the schedule, each stage's gradients are exchanged with
  the other replica's rank through the communicator and averaged;
* optimizer: Adam, lr 3e-4 (beta 0.9 / 0.999, eps 1e-5 as burn-optim).

    python examples/gpt1b/train.py --steps 10

Prints ``Step N | loss = x`` per step (as the reference's main.rs:114) and a
final JSON summary line (steps/s, loss curve, overflow count).
"""
from __future__ import annotations

import argparse
import json
import os
import struct
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

from mtorus.comm.mock import MockCommunicator  # noqa: E402
from mtorus.core.precision import Fp8Format, LossScaler  # noqa: E402
from mtorus.core.topology import MeshTorusHybrid  # noqa: E402
from mtorus.models.data import SyntheticDataLoader  # noqa: E402
from mtorus.models.gpt import GptConfig, GptModel  # noqa: E402
from mtorus.pipeline.communicator import PipelineComm  # noqa: E402
from mtorus.pipeline.placement import topology_aware_placement  # noqa: E402
from mtorus.pipeline.schedule import PipeOp, ScheduleType, build_schedule  # noqa: E402
from mtorus.pipeline.stage import StageData  # noqa: E402
from mtorus.torch_ext.autodiff_ext import enable_fp8_linears  # noqa: E402
from mtorus.torch_ext.module_ext import split_evenly  # noqa: E402


def to_stage_data(x: torch.Tensor) -> StageData:
    x2 = x.detach().reshape(-1, x.shape[-1]).float()
    return StageData(x2.reshape(-1).tolist(), x2.shape[0], x2.shape[1])


def from_stage_data(d: StageData, shape) -> torch.Tensor:
    return torch.tensor(d.values, dtype=torch.float32).reshape(shape)


def pack(grads) -> bytes:
    flat = torch.cat([g.reshape(-1) for g in grads]).float()
    return struct.pack(f"<{flat.numel()}f", *flat.tolist())


def unpack(b: bytes, like) -> list:
    flat = torch.tensor(struct.unpack(f"<{len(b) // 4}f", b), dtype=torch.float32)
    out, o = [], 0
    for g in like:
        out.append(flat[o:o + g.numel()].reshape(g.shape))
        o += g.numel()
    return out


class Replica:
    """The two pipeline stages of one data-parallel replica."""

    def __init__(self, cfg, full_state, ranks, comms, history, lr):
        self.ranks = ranks
        self.stages = []
        self.opts = []
        for s, (lo, hi) in enumerate(split_evenly(cfg.num_layers, 2)):
            m = GptModel(cfg, layers=(lo, hi), embed=s == 0, head=s == 1)
            own = m.state_dict()
            for k in own:
                g = k
                if k.startswith("blocks."):
                    j, rest = k[len("blocks."):].split(".", 1)
                    g = f"blocks.{int(j) + lo}.{rest}"
                own[k].copy_(full_state[g])
            enable_fp8_linears(m, history)
            self.stages.append(m)
            self.opts.append(torch.optim.Adam(m.parameters(), lr=lr, betas=(0.9, 0.999), eps=1e-5))
        # activations travel as E4M3 frames, gradients as E5M2 frames
        self.act = [PipelineComm(comms[r], Fp8Format.E4M3) for r in ranks]
        self.grad = [PipelineComm(comms[r], Fp8Format.E5M2) for r in ranks]

    def run_1f1b(self, ids, tgt, M, loss_scale):
        """One step of the 1F1B schedule over both stages in lock-step ticks (as the
        reference's OneF1BSchedule::execute, onef1b.rs:50-111); a stage whose input
        has not arrived yet sits the tick out.  Returns the mean loss (unscaled)."""
        sched = build_schedule(ScheduleType.OneF1B, 2, M)
        mb_ids, mb_tgt = ids.chunk(M), tgt.chunk(M)
        x_in, y_out = [dict(), dict()], [dict(), dict()]
        act_sent, grad_sent = {}, {}  # microbatch -> shape of the tensor in the mailbox
        losses = []
        idx = [0, 0]
        F_ = PipeOp.Kind.Forward
        while idx[0] < len(sched[0]) or idx[1] < len(sched[1]):
            progressed = False
            for s in range(2):
                if idx[s] >= len(sched[s]):
                    continue
                op = sched[s][idx[s]]
                m = op.microbatch
                if op.kind == F_ and s == 0:
                    y = self.stages[0].forward_stage(mb_ids[m])
                    y_out[0][m] = y
                    self.act[0].send_activations(to_stage_data(y), self.ranks[1])
                    act_sent[m] = y.shape
                elif op.kind == F_:
                    if m not in act_sent:
                        continue
                    x = from_stage_data(self.act[1].recv_activations(self.ranks[0]), act_sent.pop(m))
                    x.requires_grad_(True)
                    logits = self.stages[1].forward_stage(x)
                    x_in[1][m] = x
                    y_out[1][m] = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), mb_tgt[m].reshape(-1))
                elif s == 1:
                    loss = y_out[1].pop(m)
                    losses.append(float(loss.detach()))
                    (loss * (loss_scale / M)).backward()
                    gx = x_in[1].pop(m).grad
                    self.grad[1].send_gradients(to_stage_data(gx), self.ranks[0])
                    grad_sent[m] = gx.shape
                else:
                    if m not in grad_sent:
                        continue
                    g = from_stage_data(self.grad[0].recv_gradients(self.ranks[1]), grad_sent.pop(m))
                    y_out[0].pop(m).backward(g)
                idx[s] += 1
                progressed = True
            if not progressed:
                raise RuntimeError("1F1B schedule made no progress")
        return sum(losses) / len(losses)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--batch", type=int, default=8, help="sequences per replica per step")
    ap.add_argument("--micro-batches", type=int, default=4)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--history", type=int, default=16)
    args = ap.parse_args(argv)

    torch.manual_seed(args.seed)
    cfg = GptConfig.example_tiny()
    full = GptModel(cfg)
    state = {k: v.detach().clone() for k, v in full.state_dict().items()}

    topo = MeshTorusHybrid.new_2d(2, 2, 1)
    comms = MockCommunicator.create_world(topo.total_devices())
    place = topology_aware_placement(topo.total_devices(), topo)
    order = [r for r, _ in place]  # ranks in torus order
    replicas = [Replica(cfg, state, order[2 * r:2 * r + 2], comms, args.history, args.lr) for r in range(2)]
    scaler = LossScaler.new_dynamic(65536.0, 2000)
    loaders = [SyntheticDataLoader(args.batch, cfg.max_seq_len, cfg.vocab_size, args.steps, seed=args.seed + r,
                                   shift=True) for r in range(2)]

    curve, overflows = [], 0
    t0 = time.perf_counter()
    for step in range(args.steps):
        scale = scaler.scale_value
        for rep in replicas:
            for m in rep.stages:
                m.zero_grad(set_to_none=True)
        losses = []
        for rep, ld in zip(replicas, loaders):
            ids, tgt = ld.next()
            losses.append(rep.run_1f1b(ids, tgt, args.micro_batches, scale))
        # data parallel: each stage rank swaps gradients with its peer replica and averages
        overflow = False
        for s in range(2):
            params = [list(rep.stages[s].parameters()) for rep in replicas]
            for r, rep in enumerate(replicas):
                comms[rep.ranks[s]].send(pack([p.grad for p in params[r]]), replicas[1 - r].ranks[s])
            received = [unpack(comms[rep.ranks[s]].recv(replicas[1 - r].ranks[s]), params[r])
                        for r, rep in enumerate(replicas)]
            for r in range(2):
                for p, other in zip(params[r], received[r]):
                    p.grad = (p.grad + other) / (2.0 * scale)  # average and unscale
                    overflow |= not bool(torch.isfinite(p.grad).all())
        scaler.update(overflow)
        if overflow:
            overflows += 1
        else:
            for rep in replicas:
                for opt in rep.opts:
                    opt.step()
        loss = sum(losses) / len(losses)
        curve.append(round(loss, 6))
        print(f"Step {step + 1:3} | loss = {loss:.6f}", flush=True)
    el = time.perf_counter() - t0
    print(json.dumps({"example": "gpt1b-cpu", "steps": args.steps, "steps_per_s": round(args.steps / el, 3),
                      "tokens_per_s": round(args.steps * 2 * args.batch * cfg.max_seq_len / el, 1),
                      "loss_curve": curve, "overflows": overflows, "final_loss_scale": scaler.scale_value,
                      "world": "MockCommunicator x4 on 2x2 torus: dp2 x pp2 1F1B",
                      "fp8": "E4M3 fwd / E5M2 bwd, delayed scaling history 16"}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
