"""Training configuration with TOML round-trip.

Reference: crates/mt-training/src/config.rs.  Field names, defaults, the
validation order and the serde (externally tagged) enum encoding are kept:

    pipeline_schedule = "GPipe"            | { OneF1B = { num_stages = 8 } }
    topology_config   = "Auto"             | { Manual = { dims = [2, 2, 1] } }
    [mixed_precision] scaling_strategy = { Delayed = { history_length = 1024 } } | "Dynamic"
"""
from __future__ import annotations

import math
import tomllib
from dataclasses import dataclass, field, fields, replace
from typing import Any, Dict, Tuple

from ..core.precision import MixedPrecisionConfig


class PipelineScheduleConfig:
    @dataclass(frozen=True)
    class GPipe:
        pass

    @dataclass(frozen=True)
    class OneF1B:
        num_stages: int


class TopologyConfig:
    @dataclass(frozen=True)
    class Manual:
        dims: Tuple[int, int, int]

    @dataclass(frozen=True)
    class Auto:
        pass


class ValidationError(ValueError):
    """Carries the reference variant name and its values, e.g. ('BatchSizeTooSmall', (8, 16))."""

    _MSG = {
        "AccumulationStepsZero": "accumulation_steps must be >= 1, got {0}",
        "BatchSizeTooSmall": "batch_size ({0}) must be >= micro_batch_size ({1})",
        "BatchSizeNotDivisible": "batch_size ({0}) must be divisible by micro_batch_size ({1})",
        "EpochsZero": "epochs must be >= 1, got {0}",
        "LearningRateNonPositive": "learning_rate must be positive, got {0}",
        "MicroBatchSizeZero": "micro_batch_size must be >= 1, got {0}",
    }

    def __init__(self, kind: str, *values):
        self.kind = kind
        self.values = values
        super().__init__(self._MSG[kind].format(*values))

    def __eq__(self, other):
        return isinstance(other, ValidationError) and (self.kind, self.values) == (other.kind, other.values)

    def __hash__(self):
        return hash((self.kind, self.values))


@dataclass
class TrainingConfig:
    batch_size: int = 32
    micro_batch_size: int = 16
    accumulation_steps: int = 2
    learning_rate: float = 1e-4
    epochs: int = 10
    warmup_steps: int = 0
    mixed_precision: MixedPrecisionConfig = field(default_factory=MixedPrecisionConfig)
    pipeline_schedule: Any = field(default_factory=PipelineScheduleConfig.GPipe)
    topology_config: Any = field(default_factory=TopologyConfig.Auto)
    checkpoint_interval: int = 1000
    log_interval: int = 10
    clip_grad_norm: float = 0.0

    def validate(self) -> None:
        """Raises ValidationError; checks in the reference's order (config.rs:123-153)."""
        if self.micro_batch_size == 0:
            raise ValidationError("MicroBatchSizeZero", self.micro_batch_size)
        if self.accumulation_steps == 0:
            raise ValidationError("AccumulationStepsZero", self.accumulation_steps)
        if self.batch_size < self.micro_batch_size:
            raise ValidationError("BatchSizeTooSmall", self.batch_size, self.micro_batch_size)
        if self.batch_size % self.micro_batch_size != 0:
            raise ValidationError("BatchSizeNotDivisible", self.batch_size, self.micro_batch_size)
        if self.epochs == 0:
            raise ValidationError("EpochsZero", self.epochs)
        if not self.learning_rate > 0.0:
            raise ValidationError("LearningRateNonPositive", self.learning_rate)

    def effective_batch_size(self) -> int:
        return self.micro_batch_size * self.accumulation_steps

    def steps_per_epoch(self) -> int:
        eff = self.effective_batch_size()
        return 0 if eff == 0 else math.ceil(self.batch_size / eff)

    def replace(self, **kw) -> "TrainingConfig":
        return replace(self, **kw)

    # ------------------------------------------------------------------ serde
    def to_dict(self) -> Dict[str, Any]:
        ps = self.pipeline_schedule
        tc = self.topology_config
        return {
            "batch_size": self.batch_size, "micro_batch_size": self.micro_batch_size,
            "accumulation_steps": self.accumulation_steps, "learning_rate": float(self.learning_rate),
            "epochs": self.epochs, "warmup_steps": self.warmup_steps,
            "mixed_precision": self.mixed_precision.to_dict(),
            "pipeline_schedule": ("GPipe" if isinstance(ps, PipelineScheduleConfig.GPipe)
                                  else {"OneF1B": {"num_stages": ps.num_stages}}),
            "topology_config": ("Auto" if isinstance(tc, TopologyConfig.Auto)
                                else {"Manual": {"dims": list(tc.dims)}}),
            "checkpoint_interval": self.checkpoint_interval, "log_interval": self.log_interval,
            "clip_grad_norm": float(self.clip_grad_norm),
        }

    @staticmethod
    def from_dict(d: Dict[str, Any]) -> "TrainingConfig":
        ps = d.get("pipeline_schedule", "GPipe")
        tc = d.get("topology_config", "Auto")
        known = {f.name for f in fields(TrainingConfig)}
        unknown = set(d) - known
        if unknown:
            raise ValueError(f"unknown TrainingConfig keys: {sorted(unknown)}")
        base = TrainingConfig()
        return TrainingConfig(
            batch_size=int(d.get("batch_size", base.batch_size)),
            micro_batch_size=int(d.get("micro_batch_size", base.micro_batch_size)),
            accumulation_steps=int(d.get("accumulation_steps", base.accumulation_steps)),
            learning_rate=float(d.get("learning_rate", base.learning_rate)),
            epochs=int(d.get("epochs", base.epochs)),
            warmup_steps=int(d.get("warmup_steps", base.warmup_steps)),
            mixed_precision=MixedPrecisionConfig.from_dict(d.get("mixed_precision", {})),
            pipeline_schedule=(PipelineScheduleConfig.GPipe() if ps == "GPipe"
                               else PipelineScheduleConfig.OneF1B(int(ps["OneF1B"]["num_stages"]))),
            topology_config=(TopologyConfig.Auto() if tc == "Auto"
                             else TopologyConfig.Manual(tuple(int(x) for x in tc["Manual"]["dims"]))),
            checkpoint_interval=int(d.get("checkpoint_interval", base.checkpoint_interval)),
            log_interval=int(d.get("log_interval", base.log_interval)),
            clip_grad_norm=float(d.get("clip_grad_norm", base.clip_grad_norm)),
        )

    def to_toml(self) -> str:
        return dump_toml(self.to_dict())

    @staticmethod
    def from_toml(text: str) -> "TrainingConfig":
        return TrainingConfig.from_dict(tomllib.loads(text))

    @staticmethod
    def load(path: str) -> "TrainingConfig":
        with open(path, "rb") as f:
            return TrainingConfig.from_dict(tomllib.load(f))

    def save(self, path: str) -> None:
        with open(path, "w") as f:
            f.write(self.to_toml())


def _toml_value(v) -> str:
    if isinstance(v, bool):
        return "true" if v else "false"
    if isinstance(v, int):
        return str(v)
    if isinstance(v, float):
        r = repr(v)
        return r if any(c in r for c in ".eEn") else r + ".0"
    if isinstance(v, str):
        return '"' + v.replace("\\", "\\\\").replace('"', '\\"') + '"'
    if isinstance(v, (list, tuple)):
        return "[" + ", ".join(_toml_value(x) for x in v) + "]"
    if isinstance(v, dict):
        return "{ " + ", ".join(f"{k} = {_toml_value(x)}" for k, x in v.items()) + " }"
    raise TypeError(f"cannot encode {type(v)} as TOML")


def dump_toml(d: Dict[str, Any]) -> str:
    """Minimal TOML writer: scalars and inline tables at top level, one level of
    [section] tables for nested plain dicts."""
    top, sections = [], []
    for k, v in d.items():
        if isinstance(v, dict) and k == "mixed_precision":
            sections.append((k, v))
        else:
            top.append(f"{k} = {_toml_value(v)}")
    out = "\n".join(top) + "\n"
    for name, sec in sections:
        out += f"\n[{name}]\n" + "\n".join(f"{k} = {_toml_value(v)}" for k, v in sec.items()) + "\n"
    return out


__all__ = ["TrainingConfig", "PipelineScheduleConfig", "TopologyConfig", "ValidationError", "dump_toml"]
