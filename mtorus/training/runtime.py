"""DistributedRuntime: topology + communicator + configs + shared loss scaler.

Reference: crates/mt-training/src/runtime.rs.  ``build()`` requires a topology
(``Topology`` error) and a communicator (``Communication`` error), defaults the
configs, validates the training config (``Config`` error) and creates the loss
scaler: Dynamic scaling -> dynamic scaler (2^16, growth interval 2000),
Delayed -> static 1.0.

``init_distributed()`` is the multi-GPU entry: it joins the torch.distributed
process group from the launcher's environment (NCCL on GPUs), wraps it in an
``NcclCommunicator`` and builds a runtime over the discovered node topology.
"""
from __future__ import annotations

import logging
import os
import threading
from typing import Optional

from ..core.precision import LossScaler, MixedPrecisionConfig, ScalingStrategy
from ..core.topology import MeshTorusHybrid
from .config import TrainingConfig, ValidationError

log = logging.getLogger("mtorus.runtime")


class DistributedRuntimeError(Exception):
    pass


class _Topology(DistributedRuntimeError):
    def __init__(self, msg):
        super().__init__(f"topology error: {msg}")


class _Communication(DistributedRuntimeError):
    def __init__(self, msg):
        super().__init__(f"communication error: {msg}")


class _Pipeline(DistributedRuntimeError):
    def __init__(self, msg):
        super().__init__(f"pipeline error: {msg}")


class _Config(DistributedRuntimeError):
    def __init__(self, msg):
        super().__init__(f"configuration error: {msg}")


DistributedRuntimeError.Topology = _Topology
DistributedRuntimeError.Communication = _Communication
DistributedRuntimeError.Pipeline = _Pipeline
DistributedRuntimeError.Config = _Config


def loss_scaler_from_config(cfg: MixedPrecisionConfig) -> LossScaler:
    if isinstance(cfg.scaling_strategy, ScalingStrategy.Dynamic):
        return LossScaler.new_dynamic(65536.0, 2000)
    return LossScaler.new_static(1.0)


class SharedLossScaler:
    """Lock-protected shared loss scaler (the reference's Arc<RwLock<LossScaler>>)."""

    def __init__(self, scaler: LossScaler):
        self._scaler = scaler
        self._lock = threading.RLock()

    def read(self) -> LossScaler:
        return self._scaler

    def write(self) -> LossScaler:
        return self._scaler

    def __enter__(self):
        self._lock.acquire()
        return self._scaler

    def __exit__(self, *a):
        self._lock.release()


class DistributedRuntime:
    def __init__(self, topology, communicator, precision_config, training_config, loss_scaler):
        self.topology = topology
        self.communicator = communicator
        self.precision_config = precision_config
        self.training_config = training_config
        self.loss_scaler = loss_scaler

    @staticmethod
    def builder() -> "DistributedRuntimeBuilder":
        return DistributedRuntimeBuilder()

    def rank(self) -> int:
        return self.communicator.rank()

    def world_size(self) -> int:
        return self.communicator.world_size()

    def __repr__(self) -> str:
        return (f"DistributedRuntime {{ topology: {self.topology!r}, rank: {self.rank()}, "
                f"world_size: {self.world_size()}, precision_config: {self.precision_config!r}, "
                f"training_config: {self.training_config!r} }}")


class DistributedRuntimeBuilder:
    def __init__(self):
        self.topology: Optional[MeshTorusHybrid] = None
        self.communicator = None
        self.precision_config: Optional[MixedPrecisionConfig] = None
        self.training_config: Optional[TrainingConfig] = None

    def with_topology(self, t) -> "DistributedRuntimeBuilder":
        self.topology = t
        return self

    def with_communicator(self, c) -> "DistributedRuntimeBuilder":
        self.communicator = c
        return self

    def with_boxed_communicator(self, c) -> "DistributedRuntimeBuilder":
        return self.with_communicator(c)

    def with_precision_config(self, p) -> "DistributedRuntimeBuilder":
        self.precision_config = p
        return self

    def with_config(self, c) -> "DistributedRuntimeBuilder":
        self.training_config = c
        return self

    def build(self) -> DistributedRuntime:
        if self.topology is None:
            raise DistributedRuntimeError.Topology("topology is required")
        if self.communicator is None:
            raise DistributedRuntimeError.Communication("communicator is required")
        prec = self.precision_config or MixedPrecisionConfig()
        cfg = self.training_config or TrainingConfig()
        try:
            cfg.validate()
        except ValidationError as e:
            raise DistributedRuntimeError.Config(str(e)) from e
        scaler = SharedLossScaler(loss_scaler_from_config(prec))
        log.info("DistributedRuntime initialised: rank=%d, world_size=%d, nodes=%d",
                 self.communicator.rank(), self.communicator.world_size(), self.topology.total_nodes())
        return DistributedRuntime(self.topology, self.communicator, prec, cfg, scaler)


def init_distributed(config: Optional[TrainingConfig] = None, precision: Optional[MixedPrecisionConfig] = None,
                     backend: Optional[str] = None, timeout_s: float = 300.0) -> DistributedRuntime:
    """Join the process group of the launcher (RANK / WORLD_SIZE / MASTER_ADDR /
    MASTER_PORT) and build a runtime: one node per host, a torus of hosts."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from ..comm.nccl import DistCommunicator

    if not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        kw = {}
        if backend == "nccl":
            local = int(os.environ.get("LOCAL_RANK", "0"))
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s), **kw)
    comm = DistCommunicator()
    world = dist.get_world_size()
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    nodes = max(1, world // max(local_world, 1))
    topo = MeshTorusHybrid.new_2d(nodes, 1, max(local_world, 1))
    return (DistributedRuntime.builder().with_topology(topo).with_communicator(comm)
            .with_precision_config(precision or MixedPrecisionConfig())
            .with_config(config or TrainingConfig()).build())


__all__ = ["DistributedRuntime", "DistributedRuntimeBuilder", "DistributedRuntimeError", "SharedLossScaler",
           "loss_scaler_from_config", "init_distributed"]
