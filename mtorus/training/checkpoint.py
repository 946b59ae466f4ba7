"""Training checkpoints: save and exact restore.

The reference has no model / optimizer checkpointing: its ``checkpoint_interval``
(crates/mt-training/src/config.rs:64-65) is never read, and its "checkpoint" is
activation checkpointing.  Here a checkpoint directory holds

* ``config.toml``     -- the ``TrainingConfig`` (serde-compatible TOML), when given;
* ``rank{r}.pt``      -- one file per rank: everything that rank's trainer needs
  to continue (``trainer.state_dict()``): the fp32 master weights and
  bf16 compute copy, Adam moments and the device optimizer / loss-scale state
  block, the FP8 amax histories, scales and cursor, the global step and the torch
  CPU / CUDA RNG states;
* ``meta.json``       -- world size, step, and the list of rank files.

Each rank writes and reads only its own file (sharded optimizers keep their
shard there).  Restoring is exact; the steps after it repeat the original run up
to the fp32 summation order of atomic reductions (attention dQ, embedding
gradients), which is not fixed from run to run.  Files are written to a
temporary name and renamed, so a crash mid-save leaves the previous checkpoint
intact.
"""
from __future__ import annotations

import json
import os
from typing import Optional

import torch


def _rank_world():
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def rng_state() -> dict:
    st = {"cpu": torch.get_rng_state()}
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        st["cuda"] = torch.cuda.get_rng_state()
    return st


def set_rng_state(st: dict) -> None:
    torch.set_rng_state(st["cpu"])
    if "cuda" in st and torch.cuda.is_available():
        torch.cuda.set_rng_state(st["cuda"])


def save_checkpoint(path: str, trainer, config=None, step: Optional[int] = None) -> str:
    """Writes this rank's state (and, on rank 0, config.toml / meta.json) into ``path``."""
    rank, world = _rank_world()
    os.makedirs(path, exist_ok=True)
    sd = trainer.state_dict()
    sd["rng"] = rng_state()
    step = int(sd.get("global_step", 0) if step is None else step)
    fn = os.path.join(path, f"rank{rank}.pt")
    tmp = fn + ".tmp"
    torch.save(sd, tmp)
    os.replace(tmp, fn)
    if rank == 0:
        if config is not None:
            with open(os.path.join(path, "config.toml.tmp"), "w") as f:
                f.write(config.to_toml())
            os.replace(os.path.join(path, "config.toml.tmp"), os.path.join(path, "config.toml"))
        meta = {"world_size": world, "global_step": step, "files": [f"rank{r}.pt" for r in range(world)]}
        with open(os.path.join(path, "meta.json.tmp"), "w") as f:
            json.dump(meta, f)
        os.replace(os.path.join(path, "meta.json.tmp"), os.path.join(path, "meta.json"))
    return fn


def load_checkpoint(path: str, trainer, map_location=None):
    """Restores this rank's trainer from ``path``; returns the TrainingConfig if the
    directory has one (else None).  The world size must match the checkpoint's."""
    rank, world = _rank_world()
    meta_p = os.path.join(path, "meta.json")
    if os.path.exists(meta_p):
        meta = json.load(open(meta_p))
        if meta["world_size"] != world:
            raise ValueError(f"checkpoint was written by {meta['world_size']} ranks, this job has {world}")
    sd = torch.load(os.path.join(path, f"rank{rank}.pt"), map_location=map_location or "cpu", weights_only=False)
    trainer.load_state_dict(sd)
    if "rng" in sd:
        set_rng_state(sd["rng"])
    cfg_p = os.path.join(path, "config.toml")
    if os.path.exists(cfg_p):
        from .config import TrainingConfig

        return TrainingConfig.from_toml(open(cfg_p).read())
    return None


def maybe_save(path: str, trainer, config) -> Optional[str]:
    """Saves when ``trainer.global_step`` is a positive multiple of ``config.checkpoint_interval``."""
    k = getattr(config, "checkpoint_interval", 0)
    if k and trainer.global_step > 0 and trainer.global_step % k == 0:
        return save_checkpoint(os.path.join(path, f"step{trainer.global_step:08d}"), trainer, config)
    return None


__all__ = ["save_checkpoint", "load_checkpoint", "maybe_save", "rng_state", "set_rng_state"]
