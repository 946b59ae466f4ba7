"""Parity: crates/mt-burn/src/{fp8_ops,autodiff_ext,module_ext,optim_ext}.rs and
examples/gpt-1b/src/{model,transformer,synthetic_data}.rs tests (CPU reference path)."""
import math

import pytest
import torch

from mtorus.core.precision import Fp8Format, MixedPrecisionConfig, to_fp8
from mtorus.models import (FeedForward, GptConfig, GptModel, MultiHeadAttention, SyntheticDataLoader,
                           TransformerBlock, create_causal_mask, create_position_ids, cross_entropy_loss)
from mtorus.torch_ext import (AutodiffExt, DeviceFp8Tensor, Fp8Adam, Fp8CastFn, Fp8Gradients, Fp8Sgd, GradientHook,
                              PipelineStage, SequentialStages, cast_from_fp8, cast_to_fp8, fp8_to_torch_1d,
                              fp8_to_torch_2d, split_evenly, torch_1d_to_fp8, torch_2d_to_fp8, torch_to_fp8,
                              update_weight_fp8)
from mtorus.torch_ext.module_ext import ModuleStage, split_sequential
from mtorus.training import ParamId, param_id

E4, E5 = Fp8Format.E4M3, Fp8Format.E5M2


def rel(o, r):
    return abs(o - r) if abs(o) < 1e-8 else abs((o - r) / o)


# ---------------------------------------------------------------- fp8_ops.rs
@pytest.mark.parametrize("f,tol", [(E4, 0.07), (E5, 0.15)])
def test_roundtrip_1d_2d(f, tol):
    v = [1.0, 2.0, 3.0, 4.0, 0.5, -1.0]
    out = fp8_to_torch_1d(torch_1d_to_fp8(torch.tensor(v), f))
    assert all(rel(a, b) < tol for a, b in zip(v, out.tolist()))
    v2 = torch.tensor([[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]])
    out2 = fp8_to_torch_2d(torch_2d_to_fp8(v2, f), 2, 3)
    assert out2.shape == (2, 3) and all(rel(a, b) < tol for a, b in zip(v2.reshape(-1).tolist(), out2.reshape(-1).tolist()))


def test_fp8_preserves_format_count_and_zeros():
    assert torch_to_fp8(torch.tensor([1.0, 2.0, 3.0]), E4).format == E4
    assert torch_to_fp8(torch.tensor([1.0, 2.0, 3.0]), E5).format == E5
    assert len(torch_to_fp8(torch.tensor([1.0, 2.0, 3.0, 4.0, 5.0]), E4)) == 5
    assert all(abs(x) < 1e-6 for x in fp8_to_torch_1d(torch_to_fp8(torch.zeros(4), E4)).tolist())


def test_torch_quantiser_matches_host_codec():
    x = torch.randn(777) * 5
    for f in (E4, E5):
        a, b = torch_to_fp8(x, f), to_fp8(x.tolist(), f)
        assert a.data == b.data and a.scale == b.scale


def test_device_fp8_tensor_roundtrip():
    x = torch.randn(64, 32)
    d = DeviceFp8Tensor.quantize(x, E4)
    assert d.data.dtype == torch.float8_e4m3fn and d.dequantize().shape == x.shape
    assert ((d.dequantize() - x).abs() / x.abs().clamp_min(1e-3)).median() < 0.07
    h = d.to_host()
    assert len(h) == x.numel()


# ---------------------------------------------------------------- autodiff_ext.rs
def test_gradient_and_weight_casts():
    v = torch.tensor([0.1, 0.2, 0.3, 0.4, 0.5])
    assert all(rel(a, b) < 0.15 for a, b in zip(v.tolist(), AutodiffExt.gradient_cast_e5m2(v).tolist()))
    v = torch.tensor([[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]])
    c = AutodiffExt.gradient_cast_e5m2(v)
    assert c.numel() == 6 and all(rel(a, b) < 0.15 for a, b in zip(v.reshape(-1).tolist(), c.reshape(-1).tolist()))
    w = torch.tensor([1.0, 2.0, 3.0])
    assert all(rel(a, b) < 0.07 for a, b in zip(w.tolist(), AutodiffExt.weight_cast_e4m3(w).tolist()))
    assert AutodiffExt.weight_cast_e4m3(torch.ones(2, 3)).shape == (2, 3)
    assert GradientHook.cast_gradients_to_e5m2_preserving_shape(torch.ones(2, 2)).shape == (2, 2)
    assert GradientHook.cast_gradients_to_e5m2(torch.ones(2, 2)).shape == (2, 2)


def test_fp8_cast_function_grad_is_e5m2():
    x = torch.tensor([1.1, 2.2, 3.3], requires_grad=True)
    y = Fp8CastFn.apply(x)
    y.backward(torch.tensor([0.3, 0.7, 1.9]))
    assert torch.allclose(x.grad, AutodiffExt.gradient_cast_e5m2(torch.tensor([0.3, 0.7, 1.9])))


# ---------------------------------------------------------------- module_ext.rs
@pytest.mark.parametrize("count,n,expected", [(10, 3, [(0, 4), (4, 7), (7, 10)]), (6, 3, [(0, 2), (2, 4), (4, 6)]),
                                              (2, 5, [(0, 1), (1, 2)]), (5, 1, [(0, 5)]), (0, 3, []), (5, 0, [])])
def test_split_evenly(count, n, expected):
    assert split_evenly(count, n) == expected


def test_sequential_stages():
    ident = PipelineStage("stage_0", ModuleStage(torch.nn.Identity()))
    x = torch.randn(2, 4)
    assert torch.equal(ident.forward(x), x)
    seq = SequentialStages([PipelineStage(f"stage_{i}", ModuleStage(torch.nn.Identity())) for i in range(3)])
    assert seq.num_stages() == 3 and torch.equal(seq.forward(x), x)
    assert PipelineStage("my_stage", ModuleStage(torch.nn.Identity())).name() == "my_stage"
    assert seq.stage(0) is not None and seq.stage(2) is not None and seq.stage(3) is None
    assert seq.stage(1).name() == "stage_1"
    stages = split_sequential(torch.nn.Sequential(*[torch.nn.Linear(4, 4) for _ in range(5)]), 2)
    assert len(stages) == 2 and len(stages[0].inner.module) == 3


# ---------------------------------------------------------------- optim_ext.rs
def test_fp8_gradients():
    g = Fp8Gradients()
    assert g.is_empty()
    g.register(ParamId(1), [1.0, 2.0, 3.0])
    assert g.len() == 1 and g.remove(ParamId(1)) == [1.0, 2.0, 3.0] and g.is_empty()
    assert g.remove(ParamId(1)) is None


@pytest.mark.parametrize("f", [E4, E5])
def test_cast_roundtrip(f):
    v = [1.0, 2.0, 3.0, 0.5, -1.0]
    assert len(cast_from_fp8(cast_to_fp8(v, f))) == len(v)


def test_update_weight():
    w = torch.tensor([1.0, 2.0, 3.0])
    out = update_weight_fp8(w, cast_to_fp8([0.1, 0.2, 0.3], E5), 1.0)
    assert all(abs(o - e) < 0.1 for o, e in zip(out.tolist(), [0.9, 1.8, 2.7]))
    w = torch.tensor([[1.0, 2.0], [3.0, 4.0]])
    out = update_weight_fp8(w, cast_to_fp8([0.1] * 4, E5), 1.0)
    assert out.shape == (2, 2) and all(abs(o - e) < 0.1 for o, e in zip(out.reshape(-1).tolist(), [0.9, 1.9, 2.9, 3.9]))
    c = MixedPrecisionConfig()
    assert c.forward_format == E4 and c.backward_format == E5


def test_fp8_optimizers_step():
    m = torch.nn.Linear(3, 2)
    w0 = m.weight.detach().clone()
    g = Fp8Gradients()
    g.register(param_id(m.weight), DeviceFp8Tensor.quantize(torch.ones(2, 3), E5))
    Fp8Sgd().step_fp8(0.1, m, g)
    assert torch.allclose(m.weight, w0 - 0.1, atol=1e-3)
    g = Fp8Gradients()
    g.register(param_id(m.weight), torch_to_fp8(torch.ones(6), E5))
    w1 = m.weight.detach().clone()
    Fp8Adam().step_fp8(0.01, m, g)
    assert torch.allclose(m.weight, w1 - 0.01, atol=1e-4)  # first Adam step moves by lr * sign


# ---------------------------------------------------------------- gpt-1b example
def test_gpt_configs():
    c = GptConfig.gpt_1b()
    assert (c.vocab_size, c.d_model, c.num_layers, c.num_heads, c.d_ff, c.max_seq_len) == (50257, 2048, 24, 32, 8192, 2048)
    t = GptConfig.test_config()
    assert (t.vocab_size, t.d_model, t.num_layers, t.num_heads, t.d_ff, t.max_seq_len, t.dropout) == (
        1000, 128, 2, 4, 512, 64, 0.1)
    assert abs(GptConfig.gpt_1b_bench().num_params() / 1e9 - 1.4189) < 1e-3


def test_gpt_forward_shapes_and_finite():
    torch.manual_seed(0)
    c = GptConfig.test_config()
    m = GptModel(c).eval()
    x = torch.randint(0, c.vocab_size, (2, 8))
    out = m(x)
    assert out.shape == (2, 8, c.vocab_size) and torch.isfinite(out).all()
    assert m(torch.randint(0, c.vocab_size, (1, 4))).shape == (1, 4, c.vocab_size)
    assert m.num_layers() == 2


def test_position_ids_and_mask():
    p = create_position_ids(2, 5).reshape(-1).tolist()
    assert len(p) == 10 and all(p[i * 5 + j] == j for i in range(2) for j in range(5))
    mk = create_causal_mask(10)
    assert mk.shape == (10, 10)
    for i in range(10):
        for j in range(10):
            v = mk[i, j].item()
            assert (math.isinf(v) and v < 0) if j > i else abs(v) < 1e-6


def test_transformer_components():
    torch.manual_seed(0)
    x = torch.randn(2, 6, 64)
    mask = create_causal_mask(6).reshape(1, 1, 6, 6)
    assert MultiHeadAttention(64, 4, 0.0)(x).shape == (2, 6, 64)
    assert MultiHeadAttention(64, 4, 0.0)(x, mask).shape == (2, 6, 64)
    assert FeedForward(64, 256, 0.0)(x).shape == (2, 6, 64)
    assert TransformerBlock(64, 4, 256, 0.0)(x).shape == (2, 6, 64)
    assert TransformerBlock(64, 4, 256, 0.0)(x, mask).shape == (2, 6, 64)
    assert MultiHeadAttention(64, 4).d_head == 16
    with pytest.raises(AssertionError):
        MultiHeadAttention(65, 4)


def test_attention_is_causal():
    torch.manual_seed(0)
    mha = MultiHeadAttention(32, 2, 0.0)
    x = torch.randn(1, 5, 32)
    mask = create_causal_mask(5).reshape(1, 1, 5, 5)
    y1 = mha(x, mask)
    x2 = x.clone()
    x2[:, 3:] += 1.0
    y2 = mha(x2, mask)
    assert torch.allclose(y1[:, :3], y2[:, :3], atol=1e-6) and not torch.allclose(y1[:, 3:], y2[:, 3:])


def test_synthetic_dataloader():
    dl = SyntheticDataLoader(4, 32, 1000, 5)
    x, y = dl.next()
    assert x.shape == (4, 32) and y.shape == (4, 32) and torch.equal(x, y)
    dl = SyntheticDataLoader(2, 8, 100, 3)
    assert sum(1 for _ in dl) == 3
    dl = SyntheticDataLoader(2, 8, 100, 1)
    assert dl.next() is not None and dl.next() is None
    dl = SyntheticDataLoader(2, 8, 100, 5)
    dl.next()
    assert dl.current_batch() == 1
    dl.reset()
    assert dl.current_batch() == 0 and dl.next() is not None
    x, _ = SyntheticDataLoader(8, 64, 50, 1).next()
    assert ((x >= 0) & (x < 50)).all()
    assert SyntheticDataLoader(2, 8, 100, 0).next() is None and SyntheticDataLoader(2, 8, 100, 7).num_batches() == 7
    x, y = SyntheticDataLoader(2, 8, 100, 1, shift=True).next()
    assert x.shape == y.shape == (2, 8) and torch.equal(x[:, 1:], y[:, :-1])


def test_cross_entropy_and_training_loss_decreases():
    torch.manual_seed(0)
    c = GptConfig.example_tiny()
    c.dropout = 0.0
    m = GptModel(c)
    opt = torch.optim.Adam(m.parameters(), lr=3e-3, eps=1e-5)
    dl = SyntheticDataLoader(8, 64, c.vocab_size, 30, seed=1, shift=True)
    fixed = dl.next()
    losses = []
    for _ in range(25):
        logits = m(fixed[0])
        loss = cross_entropy_loss(logits, fixed[1])
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert abs(losses[0] - math.log(c.vocab_size)) < 1.0
    assert losses[-1] < losses[0] - 1.0


def test_native_token_loader_matches_reference_and_resumes():
    from mtorus.models.data import NativeSyntheticDataLoader, synthetic_batch_ref

    for shift, workers in ((True, 3), (False, 1)):
        dl = NativeSyntheticDataLoader(4, 16, 1000, 7, seed=5, shift=shift, depth=3, workers=workers)
        got = [tuple(t.clone() for t in b) for b in dl]
        assert len(got) == 7 and dl.next() is None and dl.current_batch() == 7
        for i, (x, y) in enumerate(got):
            rx, ry = synthetic_batch_ref(5, i, 4, 16, 1000, shift)
            assert torch.equal(x, rx) and torch.equal(y, ry)
            assert int(x.min()) >= 0 and int(x.max()) < 1000
        if shift:
            assert torch.equal(got[0][0][:, 1:], got[0][1][:, :-1])  # next-token targets
        dl.seek(4)
        x, y = dl.next()
        assert torch.equal(x, got[4][0]) and dl.current_batch() == 5
        dl.reset()
        assert torch.equal(dl.next()[0], got[0][0])


def test_native_token_loader_is_roughly_uniform():
    from mtorus.models.data import NativeSyntheticDataLoader

    dl = NativeSyntheticDataLoader(64, 256, 10, 4, seed=1)
    counts = torch.zeros(10)
    for x, _ in dl:
        counts += torch.bincount(x.reshape(-1), minlength=10).float()
    frac = counts / counts.sum()
    assert float((frac - 0.1).abs().max()) < 0.01


def test_native_token_loader_rejects_bad_arguments():
    from mtorus._ext import host
    from mtorus.models.data import NativeSyntheticDataLoader

    with pytest.raises(Exception):
        host().TokenLoader(0, 16, 100, 3, 0, False)
    dl = NativeSyntheticDataLoader(2, 8, 100, 3)
    with pytest.raises(Exception):
        dl.seek(4)  # past num_batches
    dl.seek(3)
    assert dl.next() is None
