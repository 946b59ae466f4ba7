"""Parity: crates/mt-core/src/precision/{config,fp8_tensor,quantize,scaling,loss_scale}.rs tests,
plus the codec against torch's float8 conversions."""
import math

import pytest
import torch

from mtorus.core.precision import (DelayedScaling, Fp8Format, Fp8Quantizer, Fp8Tensor, LossScaleMode, LossScaler,
                                   MasterFormat, MixedPrecisionConfig, ScalingStrategy, fp8_decode, fp8_encode,
                                   fp8_format_max, from_fp8, to_fp8, to_fp8_per_block, to_fp8_with_scale)

E4, E5 = Fp8Format.E4M3, Fp8Format.E5M2


def rel(o, r):
    return abs(o - r) if abs(o) < 1e-8 else abs((o - r) / o)


# ---------------------------------------------------------------- config.rs
def test_default_config():
    c = MixedPrecisionConfig()
    assert c.forward_format == E4 and c.backward_format == E5 and c.master_format == MasterFormat.Fp32
    assert c.scaling_strategy == ScalingStrategy.Delayed(history_length=1024)


@pytest.mark.parametrize("f", [E4, E5])
def test_format_eq(f):
    assert f == f


@pytest.mark.parametrize("f", [MasterFormat.Fp32, MasterFormat.Bf16])
def test_master_format_eq(f):
    assert f == f


def test_custom_config():
    c = MixedPrecisionConfig(E5, E4, MasterFormat.Bf16, ScalingStrategy.Dynamic())
    assert (c.forward_format, c.backward_format, c.master_format) == (E5, E4, MasterFormat.Bf16)
    assert c.scaling_strategy == ScalingStrategy.Dynamic()
    assert MixedPrecisionConfig.from_dict(c.to_dict()) == c


# ---------------------------------------------------------------- fp8_tensor.rs
def test_new_tensor_basic():
    t = Fp8Tensor([0] * 4, E4, 1.0)
    assert t.len() == 4 and not t.is_empty() and t.format == E4 and abs(t.scale - 1.0) < 1e-6
    assert t.block_scales is None and t.amax_history == []


def test_empty_tensor():
    t = Fp8Tensor([], E5, 1.0)
    assert t.len() == 0 and t.is_empty()


def test_builders():
    t = Fp8Tensor([0] * 4, E4, 1.0).with_block_scales([2.0, 4.0])
    assert t.block_scales == [2.0, 4.0]
    t = Fp8Tensor([0] * 4, E4, 1.0).with_amax_history([1.0, 2.0, 3.0])
    assert t.amax_history == [1.0, 2.0, 3.0]


def test_amax_from_history():
    assert abs(Fp8Tensor([0] * 4, E4, 1.0).with_amax_history([1.0, 5.0, 3.0]).amax() - 3.0) < 1e-6


@pytest.mark.parametrize("f", [E4, E5])
def test_amax_from_scale(f):
    assert abs(Fp8Tensor([0] * 4, f, 208.0).amax() - fp8_format_max(f) / 208.0) < 1e-3


def test_tensor_clone_equality():
    t = Fp8Tensor([1, 2, 3], E4, 2.0).with_amax_history([4.0])
    assert t == t.clone()


# ---------------------------------------------------------------- quantize.rs
@pytest.mark.parametrize("f", [E4, E5])
def test_roundtrip_zeros(f):
    assert all(abs(v) < 1e-6 for v in from_fp8(to_fp8([0.0, 0.0, 0.0], f)))


@pytest.mark.parametrize("f,tol", [(E4, 0.07), (E5, 0.15)])
@pytest.mark.parametrize("values", [[0.25, 0.5, 0.75, 1.0, 1.5, 2.0, 3.0, 4.0], [0.1, 0.3, 0.7, 1.3, 2.7, 5.0]])
def test_roundtrip_values(f, tol, values):
    for o, r in zip(values, from_fp8(to_fp8(values, f))):
        assert rel(o, r) < tol, (o, r)


def test_roundtrip_negative_values():
    v = [-1.0, -2.0, -0.5, 0.5, 1.0, 2.0]
    for o, r in zip(v, from_fp8(to_fp8(v, E4))):
        assert rel(o, r) < 0.07


def test_roundtrip_preserves_shape():
    t = to_fp8([1.0, 2.0, 3.0, 4.0, 5.0], E4)
    assert t.len() == 5 and len(from_fp8(t)) == 5


def test_to_fp8_sets_amax_history():
    t = to_fp8([1.0, -3.0, 2.0], E4)
    assert len(t.amax_history) == 1 and abs(t.amax_history[0] - 3.0) < 1e-6


def test_to_fp8_computes_scale():
    assert abs(to_fp8([1.0, 2.0, 4.0], E4).scale - 416.0 / 4.0) < 1e-3


def test_per_block_quantization():
    v = [1.0, 2.0, 100.0, 200.0]
    t = to_fp8_per_block(v, E4, 2)
    assert t.block_scales is not None and len(t.block_scales) == 2
    for o, r in zip(v, from_fp8(t)):
        assert rel(o, r) < 0.07


def test_per_block_better_than_per_tensor():
    v = [1.0, 2.0, 100.0, 200.0]
    te = max(rel(o, r) for o, r in zip(v, from_fp8(to_fp8(v, E4))))
    be = max(rel(o, r) for o, r in zip(v, from_fp8(to_fp8_per_block(v, E4, 2))))
    assert be <= te + 0.01


def test_per_block_ragged_tail_uses_true_block_size():
    # len 9, block 4 -> blocks of 4, 4, 1 (the reference would infer ceil(9/3) = 3)
    v = [1.0, 2.0, 3.0, 4.0, 10.0, 20.0, 30.0, 40.0, 1000.0]
    for o, r in zip(v, from_fp8(to_fp8_per_block(v, E4, 4))):
        assert rel(o, r) < 0.07


def test_to_fp8_with_custom_scale():
    t = to_fp8_with_scale([1.0, 2.0, 3.0], E4, 100.0)
    assert abs(t.scale - 100.0) < 1e-6 and t.len() == 3


def test_quantizer_trait_impl():
    assert len(Fp8Quantizer.from_fp8(Fp8Quantizer.to_fp8([1.0, 2.0, 3.0], E4))) == 3


@pytest.mark.parametrize("f,dt", [(E4, torch.float8_e4m3fn), (E5, torch.float8_e5m2)])
def test_codec_matches_torch_float8(f, dt):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, generator=g) * torch.logspace(-6, 2, 4096)
    x = x.clamp(-400, 400)
    codes = [fp8_encode(float(v), f) for v in x]
    ref = x.to(dt).view(torch.uint8).tolist()
    assert codes == ref
    for c in range(256):
        a, b = fp8_decode(c, f), float(torch.tensor([c], dtype=torch.uint8).view(dt).float())
        assert (math.isnan(a) and math.isnan(b)) or a == b


def test_codec_saturates():
    assert fp8_decode(fp8_encode(1e6, E4), E4) == 448.0 and fp8_decode(fp8_encode(-1e6, E4), E4) == -448.0
    assert fp8_decode(fp8_encode(1e9, E5), E5) == 57344.0


# ---------------------------------------------------------------- scaling.rs
def test_delayed_scaling_ring():
    ds = DelayedScaling(4)
    assert ds.amax_history == [0.0] * 4 and ds.current_amax() == 0.0
    ds = DelayedScaling(3)
    for a in (1.0, 2.0, 3.0):
        ds.update(a)
    assert ds.amax_history == [1.0, 2.0, 3.0] and ds.current_amax() == 3.0
    ds.update(4.0)
    assert ds.amax_history == [4.0, 2.0, 3.0] and ds.current_amax() == 4.0
    ds = DelayedScaling(2)
    for a in (10.0, 5.0, 1.0, 2.0):
        ds.update(a)
    assert ds.amax_history == [1.0, 2.0] and ds.current_amax() == 2.0


@pytest.mark.parametrize("f,mx", [(E4, 416.0), (E5, 49152.0)])
def test_compute_scale(f, mx):
    assert fp8_format_max(f) == mx
    assert DelayedScaling(4).compute_scale(f) == 1.0
    ds = DelayedScaling(4)
    ds.update(2.0)
    assert abs(ds.compute_scale(f) - mx / 2.0) < 1e-3


def test_scale_uses_max_amax_from_history():
    ds = DelayedScaling(4)
    for a in (1.0, 5.0, 3.0):
        ds.update(a)
    assert abs(ds.compute_scale(E4) - 416.0 / 5.0) < 1e-3


def test_delayed_scaling_convergence():
    ds = DelayedScaling(4)
    scales = []
    for a in (1.0, 2.0, 4.0, 8.0, 4.0, 2.0, 1.0, 0.5):
        ds.update(a)
        scales.append(ds.compute_scale(E4))
    assert scales[3] < scales[0] and scales[7] > scales[3]


def test_delayed_scaling_clone_and_zero_history():
    ds = DelayedScaling(4)
    ds.update(1.0)
    ds.update(2.0)
    assert ds == ds.clone()
    with pytest.raises(ValueError):
        DelayedScaling(0)


# ---------------------------------------------------------------- loss_scale.rs
def test_scaler_initial_values():
    s = LossScaler.new_dynamic(65536.0, 2000)
    assert s.scale() == 65536.0 and s.mode == LossScaleMode.Dynamic and s.growth_interval == 2000
    assert s.growth_counter == 0
    s = LossScaler.new_static(1024.0)
    assert s.scale() == 1024.0 and s.mode == LossScaleMode.Static


def test_overflow_halves_and_resets():
    s = LossScaler.new_dynamic(1024.0, 100)
    s.update(True)
    assert s.scale() == 512.0
    s = LossScaler.new_dynamic(1024.0, 100)
    for _ in range(50):
        s.update(False)
    assert s.growth_counter == 50
    s.update(True)
    assert s.growth_counter == 0


def test_growth_doubles_after_interval():
    s = LossScaler.new_dynamic(1024.0, 4)
    for _ in range(3):
        s.update(False)
        assert s.scale() == 1024.0
    s.update(False)
    assert s.scale() == 2048.0 and s.growth_counter == 0


def test_floor_static_reset():
    s = LossScaler.new_dynamic(1.0, 100)
    s.update(True)
    assert s.scale() == 1.0
    s = LossScaler.new_static(1024.0)
    s.update(True)
    assert s.scale() == 1024.0
    for _ in range(100):
        s.update(False)
    assert s.scale() == 1024.0
    s = LossScaler.new_dynamic(1024.0, 100)
    s.update(True)
    s.update(True)
    s.reset(65536.0)
    assert s.scale() == 65536.0 and s.growth_counter == 0


@pytest.mark.parametrize("seq,expected", [((False, False, False, False), 2048.0), ((True, False, False, False), 1024.0)])
def test_loss_scaling_scenarios(seq, expected):
    s = LossScaler.new_dynamic(1024.0, 3)
    for o in seq:
        s.update(o)
    assert s.scale() == expected


def test_overflow_behavior_sequence():
    s = LossScaler.new_dynamic(65536.0, 2)
    s.update(True)
    assert s.scale() == 32768.0
    s.update(False)
    assert s.scale() == 32768.0
    s.update(False)
    assert s.scale() == 65536.0


def test_scaler_clone_equality():
    s = LossScaler.new_dynamic(1024.0, 100)
    assert s == s.clone()


def test_fp8_state_slots_capacity_and_checkpoint_round_trip():
    """Host bookkeeping of the device delayed-scaling state (mtorus.ops.fp8.Fp8State),
    on CPU tensors: one slot per tensor role in first-use order with the role's format
    maximum, a clear error past the capacity, and a state_dict that restores roles,
    formats, histories, scales and the ring cursor into a fresh state."""
    from mtorus.ops import fp8 as F8

    st = F8.Fp8State("cpu", history=4, capacity=3)
    assert st.recipe == "tensor"
    assert st.slot("L0.qkv_in", F8.E4M3) == 0 and st.slot("L0.out_grad", F8.E5M2) == 1
    assert st.slot("L0.qkv_in", F8.E4M3) == 0  # idempotent
    assert float(st.fmax[0]) == 416.0 and float(st.fmax[1]) == 49152.0
    st.slot("L0.ffn1_in", F8.E4M3)
    with pytest.raises(RuntimeError, match="capacity"):
        st.slot("L0.one_too_many", F8.E4M3)
    st.hist[:3] = torch.arange(12, dtype=torch.float32).view(3, 4)
    st.scale[:3] = torch.tensor([2.0, 4.0, 8.0])
    st.inv[:3] = 1.0 / st.scale[:3]
    st.cursor_dev.fill_(2)
    st.first_step = False
    sd = st.state_dict()
    fresh = F8.Fp8State("cpu", history=4, capacity=8)
    fresh.load_state_dict(sd)
    assert fresh.names == st.names and fresh.fmts == st.fmts
    assert torch.equal(fresh.hist[:3], st.hist[:3]) and torch.equal(fresh.scale[:3], st.scale[:3])
    assert torch.equal(fresh.inv[:3], st.inv[:3]) and int(fresh.cursor_dev) == 2 and fresh.cursor == 2
    assert not fresh.first_step
