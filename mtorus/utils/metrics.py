"""Per-step training metrics as JSON lines, plus optional NVTX ranges.

Reference: StepMetrics{loss, learning_rate, step, overflow, grad_norm} and
TrainingMetrics{avg_loss, total_steps, total_time_secs, overflow_count}
(crates/mt-training/src/step.rs:16-43), printed by the example as
``Step N | loss = x``.  Here each step becomes one JSON object (those fields plus
tokens/s, step time and the loss scale) appended to a file, and ``summary()``
returns the TrainingMetrics counterpart.  ``nvtx_range(name)`` marks host-side
regions for a timeline profiler when ``MTORUS_NVTX=1``.
"""
from __future__ import annotations

import contextlib
import json
import os
import time
from typing import Optional


class MetricsLogger:
    def __init__(self, path: Optional[str] = None, tokens_per_step: int = 0, echo: bool = False):
        self.path = path
        self.tokens_per_step = tokens_per_step
        self.echo = echo
        self.f = open(path, "a") if path else None
        self.n = 0
        self.loss_sum = 0.0
        self.overflows = 0
        self.t0 = time.perf_counter()
        self._last = self.t0

    def log(self, step: int, loss: float, lr: float, grad_norm: float = float("nan"), overflow: bool = False,
            loss_scale: float = 1.0, **extra) -> dict:
        now = time.perf_counter()
        dt = now - self._last
        self._last = now
        rec = {"step": step, "loss": loss, "learning_rate": lr, "grad_norm": grad_norm, "overflow": overflow,
               "loss_scale": loss_scale, "step_time_s": round(dt, 6)}
        if self.tokens_per_step and dt > 0:
            rec["tokens_per_s"] = round(self.tokens_per_step / dt, 1)
        rec.update(extra)
        self.n += 1
        self.loss_sum += loss
        self.overflows += int(bool(overflow))
        if self.f:
            self.f.write(json.dumps(rec) + "\n")
            self.f.flush()
        if self.echo:
            print(f"Step {step:3} | loss = {loss:.6f}", flush=True)
        return rec

    def summary(self) -> dict:
        """TrainingMetrics{avg_loss, total_steps, total_time_secs, overflow_count}."""
        return {"avg_loss": self.loss_sum / max(self.n, 1), "total_steps": self.n,
                "total_time_secs": time.perf_counter() - self.t0, "overflow_count": self.overflows}

    def close(self) -> None:
        if self.f:
            self.f.close()
            self.f = None


@contextlib.contextmanager
def nvtx_range(name: str):
    if os.environ.get("MTORUS_NVTX") == "1":
        import torch

        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


__all__ = ["MetricsLogger", "nvtx_range"]
