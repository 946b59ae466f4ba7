"""Parity: crates/mt-training/src/{config,runtime,accumulator,step}.rs tests."""
import math

import pytest
import torch

from mtorus.comm import MockCommunicator
from mtorus.core.precision import Fp8Format, LossScaler, MixedPrecisionConfig, ScalingStrategy
from mtorus.core.topology import MeshTorusHybrid
from mtorus.training import (Counter, DistributedRuntime, DistributedRuntimeBuilder, DistributedRuntimeError,
                             GradientAccumulator, GradientsParams, ParamId, PipelineScheduleConfig, StepError,
                             StepMetrics, TopologyConfig, TrainingConfig, TrainingError, TrainingMetrics,
                             ValidationError, apply_clip_norm, check_overflow_values, clip_grad_norm,
                             compute_grad_norm, list_param_ids, train_step, training_loop)
from mtorus.training.step import warmup_lr


# ---------------------------------------------------------------- config.rs
def test_default_config():
    c = TrainingConfig()
    assert (c.batch_size, c.micro_batch_size, c.accumulation_steps, c.epochs, c.warmup_steps) == (32, 16, 2, 10, 0)
    assert abs(c.learning_rate - 1e-4) < 1e-10
    assert c.pipeline_schedule == PipelineScheduleConfig.GPipe() and c.topology_config == TopologyConfig.Auto()
    assert (c.checkpoint_interval, c.log_interval, c.clip_grad_norm) == (1000, 10, 0.0)
    c.validate()


@pytest.mark.parametrize("kw,err", [
    (dict(accumulation_steps=0), ValidationError("AccumulationStepsZero", 0)),
    (dict(micro_batch_size=0), ValidationError("MicroBatchSizeZero", 0)),
    (dict(batch_size=8, micro_batch_size=16), ValidationError("BatchSizeTooSmall", 8, 16)),
    (dict(batch_size=30, micro_batch_size=16), ValidationError("BatchSizeNotDivisible", 30, 16)),
    (dict(learning_rate=0.0), ValidationError("LearningRateNonPositive", 0.0)),
    (dict(epochs=0), ValidationError("EpochsZero", 0)),
])
def test_validation_errors(kw, err):
    with pytest.raises(ValidationError) as e:
        TrainingConfig(**kw).validate()
    assert e.value == err


def test_effective_and_steps_per_epoch():
    assert TrainingConfig(micro_batch_size=8, accumulation_steps=4).effective_batch_size() == 32
    assert TrainingConfig().steps_per_epoch() == 1


def test_custom_valid_config():
    c = TrainingConfig(batch_size=128, micro_batch_size=32, accumulation_steps=4, learning_rate=1e-3, epochs=50,
                       warmup_steps=100, pipeline_schedule=PipelineScheduleConfig.OneF1B(4),
                       topology_config=TopologyConfig.Manual((2, 2, 1)))
    c.validate()
    assert c.effective_batch_size() == 128


def test_serialization_roundtrip():
    c = TrainingConfig()
    assert TrainingConfig.from_toml(c.to_toml()) == c
    c = TrainingConfig(batch_size=256, micro_batch_size=64, accumulation_steps=4, learning_rate=5e-4, epochs=100)
    d = TrainingConfig.from_toml(c.to_toml())
    assert d == c and d.batch_size == 256 and d.epochs == 100
    c = TrainingConfig(pipeline_schedule=PipelineScheduleConfig.OneF1B(8), topology_config=TopologyConfig.Manual((2, 4, 1)),
                       mixed_precision=MixedPrecisionConfig(scaling_strategy=ScalingStrategy.Dynamic()))
    s = c.to_toml()
    assert "OneF1B = { num_stages = 8 }" in s and "Manual = { dims = [2, 4, 1] }" in s
    assert TrainingConfig.from_toml(s) == c


def test_validation_passes_with_manual_topology():
    TrainingConfig(topology_config=TopologyConfig.Manual((4, 4, 1))).validate()


def test_enum_equality():
    assert PipelineScheduleConfig.GPipe() == PipelineScheduleConfig.GPipe()
    assert PipelineScheduleConfig.GPipe() != PipelineScheduleConfig.OneF1B(4)
    assert PipelineScheduleConfig.OneF1B(4) == PipelineScheduleConfig.OneF1B(4)
    assert PipelineScheduleConfig.OneF1B(4) != PipelineScheduleConfig.OneF1B(8)
    assert TopologyConfig.Auto() == TopologyConfig.Auto()
    assert TopologyConfig.Manual((2, 2, 1)) == TopologyConfig.Manual((2, 2, 1))
    assert TopologyConfig.Auto() != TopologyConfig.Manual((2, 2, 1))


# ---------------------------------------------------------------- runtime.rs
def _topo():
    return MeshTorusHybrid.new_2d(2, 2, 2)


def _cfg():
    return TrainingConfig(batch_size=32, micro_batch_size=16, accumulation_steps=2)


def _comm(n=4):
    return MockCommunicator.create_world(n)[0]


def test_builder():
    b = DistributedRuntimeBuilder()
    assert b.topology is None and b.communicator is None
    assert DistributedRuntimeBuilder().with_topology(_topo()).topology.total_nodes() == 4


def test_build_success_and_errors():
    rt = DistributedRuntime.builder().with_topology(_topo()).with_communicator(_comm()).with_config(_cfg()).build()
    assert rt.rank() == 0 and rt.world_size() == 4
    with pytest.raises(DistributedRuntimeError.Topology):
        DistributedRuntime.builder().with_communicator(_comm()).with_config(_cfg()).build()
    with pytest.raises(DistributedRuntimeError.Communication):
        DistributedRuntime.builder().with_topology(_topo()).with_config(_cfg()).build()
    with pytest.raises(DistributedRuntimeError.Config):
        DistributedRuntime.builder().with_topology(_topo()).with_communicator(_comm()).with_config(
            TrainingConfig(accumulation_steps=0)).build()


def test_world_size_boxed_and_precision():
    rt = DistributedRuntime.builder().with_topology(_topo()).with_communicator(_comm(8)).with_config(_cfg()).build()
    assert rt.world_size() == 8 and rt.rank() == 0
    rt = DistributedRuntime.builder().with_topology(_topo()).with_boxed_communicator(_comm(2)).with_config(_cfg()).build()
    assert rt.world_size() == 2
    rt = DistributedRuntime.builder().with_topology(_topo()).with_communicator(_comm()).with_config(_cfg()).build()
    assert rt.precision_config == MixedPrecisionConfig()
    p = MixedPrecisionConfig(forward_format=Fp8Format.E5M2, backward_format=Fp8Format.E4M3)
    rt = DistributedRuntime.builder().with_topology(_topo()).with_communicator(_comm()).with_precision_config(p) \
        .with_config(_cfg()).build()
    assert rt.precision_config.forward_format == Fp8Format.E5M2


def test_loss_scaler_and_debug():
    rt = DistributedRuntime.builder().with_topology(_topo()).with_communicator(_comm()).with_config(_cfg()).build()
    assert abs(rt.loss_scaler.read().scale() - 1.0) < 1e-6
    s1, s2 = rt.loss_scaler, rt.loss_scaler
    assert s1.read().scale() == s2.read().scale()
    d = repr(rt)
    assert "DistributedRuntime" in d and "rank: 0" in d and "world_size: 4" in d
    dyn = MixedPrecisionConfig(scaling_strategy=ScalingStrategy.Dynamic())
    rt = DistributedRuntime.builder().with_topology(_topo()).with_communicator(_comm()).with_precision_config(dyn) \
        .with_config(_cfg()).build()
    assert rt.loss_scaler.read().scale() == 65536.0 and rt.loss_scaler.read().growth_interval == 2000


def test_multiple_builders_independent():
    a = DistributedRuntime.builder().with_topology(_topo()).with_communicator(_comm()).with_config(_cfg()).build()
    b = DistributedRuntime.builder().with_topology(MeshTorusHybrid.new_2d(3, 3, 2)).with_communicator(_comm(2)) \
        .with_config(_cfg()).build()
    assert a.world_size() == 4 and b.world_size() == 2


# ---------------------------------------------------------------- accumulator.rs
def test_accumulator_basics():
    acc = GradientAccumulator()
    assert acc.step_count() == 0 and not acc.raw_grads()
    acc.register(ParamId(1), torch.tensor([0.5, 0.2, -0.1]))
    assert acc.step_count() == 1 and len(acc.raw_grads()) == 1
    acc = GradientAccumulator()
    acc.register(ParamId(1), torch.tensor([0.1, 0.2]))
    acc.register(ParamId(2), torch.tensor([0.3, 0.4, 0.5]))
    assert acc.step_count() == 2 and len(acc.raw_grads()) == 2


def test_accumulator_sums_reset_and_effective_batch():
    acc = GradientAccumulator()
    acc.register(ParamId(1), torch.tensor([1.0, 2.0]))
    acc.register(ParamId(1), torch.tensor([3.0, 4.0]))
    assert acc.raw_grads()[ParamId(1)].tolist() == [4.0, 6.0] and acc.step_count() == 2
    acc.reset()
    assert acc.step_count() == 0 and not acc.raw_grads()
    assert acc.effective_batch_size(16) == 0
    for _ in range(4):
        acc.register(ParamId(1), torch.tensor([1.0]))
    assert acc.effective_batch_size(16) == 64 and acc.effective_batch_size(32) == 128


def test_into_gradients_and_drain():
    acc = GradientAccumulator()
    acc.register(ParamId(1), torch.tensor([0.5, -0.5]))
    gp = acc.into_gradients()
    assert len(gp) == 1 and not acc.raw_grads() and acc.step_count() == 1
    m = torch.nn.Linear(4, 2)
    ids = list_param_ids(m)
    acc = GradientAccumulator()
    for _ in range(3):
        gp = GradientsParams()
        for i, pid in enumerate(ids):
            gp.register(pid, torch.tensor([(i + 1) * 0.5]))
        acc.drain_from(gp, ids)
    assert acc.step_count() == 3
    for i, pid in enumerate(ids):
        assert abs(acc.raw_grads()[pid][0].item() - (i + 1) * 0.5 * 3) < 1e-5
    acc = GradientAccumulator()
    gp = GradientsParams()
    gp.register(ParamId(1), torch.tensor([3.0, 4.0]))
    assert abs(acc.drain_from(gp, [ParamId(1)]) - 5.0) < 1e-5


def test_accumulate_after_reset_register_values_debug_device():
    acc = GradientAccumulator()
    acc.register(ParamId(1), torch.tensor([10.0]))
    acc.reset()
    acc.register(ParamId(1), torch.tensor([5.0]))
    assert acc.step_count() == 1 and acc.raw_grads()[ParamId(1)].tolist() == [5.0]
    assert "GradientAccumulator" in repr(acc) and "count: 1" in repr(acc)
    acc = GradientAccumulator()
    acc.register_values(ParamId(1), [1.0, 2.0])
    acc.register_values(ParamId(1), [3.0, 4.0])
    assert acc.raw_grads()[ParamId(1)].tolist() == [4.0, 6.0] and acc.step_count() == 2
    assert GradientAccumulator("cpu").device == torch.device("cpu")


# ---------------------------------------------------------------- step.rs
def test_compute_grad_norm():
    assert abs(compute_grad_norm([3.0, 4.0]) - 5.0) < 1e-6
    assert abs(compute_grad_norm([0.0, 0.0, 0.0])) < 1e-6
    assert abs(compute_grad_norm([-3.0, -4.0]) - 5.0) < 1e-6
    assert abs(compute_grad_norm([])) < 1e-6


@pytest.mark.parametrize("g,mx,n,g0", [([1.0, 2.0, 3.0], 10.0, 3.741657, 1.0), ([10.0, 0.0, 0.0], 5.0, 10.0, 5.0),
                                       ([0.0, 0.0], 1.0, 0.0, 0.0), ([6.0, 8.0], 10.0, 10.0, 6.0)])
def test_clip(g, mx, n, g0):
    t = torch.tensor(g)
    assert abs(clip_grad_norm(t, mx) - n) < 1e-4 and abs(t[0].item() - g0) < 1e-6


def test_clip_mixed_sign():
    t = torch.tensor([3.0, -4.0, 0.0])
    assert abs(clip_grad_norm(t, 2.5) - 5.0) < 1e-6 and abs(t[0] - 1.5) < 1e-6 and abs(t[1] + 2.0) < 1e-6


def test_check_overflow():
    n, o = check_overflow_values({ParamId(1): torch.tensor([1.0, 2.0])})
    assert not o and n > 0.0
    _, o = check_overflow_values({ParamId(1): torch.tensor([float("nan")])})
    assert o


def test_metrics_structs_and_errors():
    m = StepMetrics(1.0, 1e-4, 0, False, 0.5)
    assert abs(m.loss - 1.0) < 1e-6 and abs(m.learning_rate - 1e-4) < 1e-10 and m.step == 0
    t = TrainingMetrics(2.5, 100, 10.0, 0)
    assert abs(t.avg_loss - 2.5) < 1e-6 and t.total_steps == 100
    assert str(StepError.Overflow()) == "gradient overflow detected, skipping step"
    assert str(StepError.ShapeMismatch("x")) == "gradient shape mismatch: x"
    assert str(StepError.Internal("y")) == "step error: y"
    assert str(TrainingError.EmptyDataloader()) == "dataloader is empty"
    assert "step 5" in str(TrainingError.StepError(5, StepError.Overflow()))


def _grads(m, vals):
    gp = GradientsParams()
    for pid in list_param_ids(m):
        gp.register(pid, torch.tensor(vals))
    return gp


def test_train_step_overflow_error():
    m = torch.nn.Linear(4, 2)
    acc, sc, gs = GradientAccumulator(), LossScaler.new_dynamic(65536.0, 2000), Counter(0)
    with pytest.raises(StepError.Overflow):
        train_step(_grads(m, [float("nan")]), 1.0, TrainingConfig(), acc, sc, gs, m)
    assert sc.scale() == 32768.0 and acc.step_count() == 0


def test_train_step_no_opt_step_early_and_accumulates():
    m = torch.nn.Linear(4, 2)
    cfg = TrainingConfig(accumulation_steps=4)
    acc, sc, gs = GradientAccumulator(), LossScaler.new_static(1.0), Counter(0)
    r = train_step(_grads(m, [0.1, 0.2, 0.3]), 1.5, cfg, acc, sc, gs, m)
    assert abs(r.loss - 1.5) < 1e-6 and gs.value == 0 and acc.step_count() == 1
    cfg = TrainingConfig(accumulation_steps=3)
    acc, gs = GradientAccumulator(), Counter(0)
    for _ in range(3):
        train_step(_grads(m, [0.1, 0.2, 0.3]), 1.0, cfg, acc, sc, gs, m)
    assert gs.value == 1
    acc.into_gradients()
    assert not acc.raw_grads() and acc.step_count() == 3
    acc.reset()
    assert acc.step_count() == 0


def test_apply_clip_norm_fn():
    acc = GradientAccumulator()
    acc.register_values(ParamId(1), [30.0, 40.0])
    apply_clip_norm(acc, 10.0)
    assert abs(acc.raw_grads()[ParamId(1)][0].item() - 6.0) < 1e-5
    acc = GradientAccumulator()
    acc.register_values(ParamId(1), [5.0])
    apply_clip_norm(acc, 10.0)
    assert abs(acc.raw_grads()[ParamId(1)][0].item() - 5.0) < 1e-6


def test_lr_warmup():
    cfg = TrainingConfig(learning_rate=1e-3, warmup_steps=100)
    assert abs(warmup_lr(cfg, 0)) < 1e-10 and abs(warmup_lr(cfg, 50) - 5e-4) < 1e-10
    assert abs(warmup_lr(cfg, 100) - 1e-3) < 1e-10
    cfg = TrainingConfig(learning_rate=1e-4)
    assert all(abs(warmup_lr(cfg, s) - 1e-4) < 1e-10 for s in range(10))


def test_training_loop_scaffold():
    t = training_loop(None, [(1, 1)] * 3, TrainingConfig())
    assert t.total_steps == 3
    with pytest.raises(TrainingError.EmptyDataloader):
        training_loop(None, [], TrainingConfig())


def test_gpt1b_cpu_example_runs_dp_pp_fp8(capsys):
    """The CPU example (MockCommunicator x4 on a 2x2 torus, DP2 x PP2 1F1B, FP8
    delayed scaling, dynamic loss scale) trains two steps with finite losses."""
    import importlib.util
    import json
    import os

    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "examples", "gpt1b", "train.py")
    spec = importlib.util.spec_from_file_location("gpt1b_example", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.main(["--steps", "2"]) == 0
    out = capsys.readouterr().out.strip().splitlines()
    assert out[0].startswith("Step   1 | loss = ")
    summary = json.loads(out[-1])
    assert summary["overflows"] == 0 and len(summary["loss_curve"]) == 2
    assert all(6.0 < v < 8.0 for v in summary["loss_curve"])


def test_checkpoint_files_roundtrip_cpu(tmp_path):
    """save / load on a host-only trainer: config TOML, per-rank file, meta, RNG state."""
    import json

    import torch

    from mtorus.training.checkpoint import load_checkpoint, maybe_save, save_checkpoint
    from mtorus.training.config import TrainingConfig

    class Toy:
        def __init__(self):
            self.w = torch.zeros(4)
            self.global_step = 0

        def state_dict(self):
            return {"w": self.w.clone(), "global_step": self.global_step}

        def load_state_dict(self, d):
            self.w = d["w"].clone()
            self.global_step = d["global_step"]

    t = Toy()
    t.w += 3.0
    t.global_step = 7
    cfg = TrainingConfig(checkpoint_interval=7)
    torch.manual_seed(5)
    p = maybe_save(str(tmp_path), t, cfg)
    assert p is not None and p.endswith("rank0.pt")
    r1 = torch.rand(3)
    u = Toy()
    back = load_checkpoint(str(tmp_path / "step00000007"), u)
    assert back == cfg and u.global_step == 7 and torch.equal(u.w, torch.full((4,), 3.0))
    assert torch.equal(torch.rand(3), r1)  # RNG restored to the save point
    meta = json.load(open(tmp_path / "step00000007" / "meta.json"))
    assert meta == {"world_size": 1, "global_step": 7, "files": ["rank0.pt"]}
    t.global_step = 8
    assert maybe_save(str(tmp_path), t, cfg) is None
    save_checkpoint(str(tmp_path / "x"), t)


def test_train_cli_set_overrides():
    import importlib.util
    import os

    from mtorus.training.config import PipelineScheduleConfig, TrainingConfig

    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "examples", "gpt1b",
                        "train_gpu.py")
    spec = importlib.util.spec_from_file_location("train_gpu", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    d = mod.parse_set(["learning_rate=3e-4", "pipeline_schedule={OneF1B={num_stages=4}}",
                       "mixed_precision.scaling_strategy=\"Dynamic\"", "checkpoint_interval=100"],
                      TrainingConfig().to_dict())
    tc = TrainingConfig.from_dict(d)
    assert tc.learning_rate == 3e-4 and tc.checkpoint_interval == 100
    assert tc.pipeline_schedule == PipelineScheduleConfig.OneF1B(4)
    assert tc.mixed_precision.to_dict()["scaling_strategy"] == "Dynamic"


def test_metrics_logger_jsonl_and_summary(tmp_path):
    import json

    from mtorus.utils.metrics import MetricsLogger, nvtx_range

    p = tmp_path / "m.jsonl"
    log = MetricsLogger(str(p), tokens_per_step=1000)
    with nvtx_range("step"):
        log.log(1, 7.0, 3e-4, grad_norm=1.5, overflow=False, loss_scale=65536.0)
    log.log(2, 5.0, 3e-4, overflow=True, extra_key=3)
    s = log.summary()
    log.close()
    recs = [json.loads(x) for x in open(p)]
    assert [r["step"] for r in recs] == [1, 2] and recs[0]["grad_norm"] == 1.5 and recs[1]["extra_key"] == 3
    assert recs[0]["loss_scale"] == 65536.0 and "tokens_per_s" in recs[0]
    assert s["total_steps"] == 2 and s["avg_loss"] == 6.0 and s["overflow_count"] == 1


def test_fused_model_builds_the_reference_dropout_state():
    """The reference config's p = 0.1 gives the fused path a Philox dropout state (the
    GPU tests in test_dropout.py check the masks); p = 0 gives none."""
    from mtorus.models.gpt import GptConfig, GptModel

    cfg = GptConfig(vocab_size=64, d_model=32, num_layers=1, num_heads=2, d_ff=64, max_seq_len=16, dropout=0.1)
    m = GptModel(cfg)
    m.flatten("cpu")
    st = m.enable_dropout(seed=4)
    assert st is not None and st.p == 0.1 and st.thr16 == 6554
    cfg.dropout = 0.0
    m2 = GptModel(cfg)
    m2.flatten("cpu")
    assert m2.enable_dropout() is None
