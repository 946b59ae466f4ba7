"""Dropout of the fused GPT path: Philox4x32-10 masks drawn inside the kernels.

CPU: the NumPy Philox restatement reproduces the published known-answer vectors
and the mask keeps 1 - p of the elements.  GPU: every kernel that draws a mask
(standalone apply, embedding, the three GEMM epilogue modes, attention forward and
backward) matches a PyTorch fp32 computation that uses the oracle's mask."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from mtorus.ops.dropout import DropoutState, keep_mask_ref, philox4x32_10, threshold16


def test_philox_known_answer_vectors():
    """Philox4x32-10 known-answer tests (Salmon et al., SC'11; Random123 kat_vectors)."""
    def run(c, k):
        return [int(x[0]) for x in philox4x32_10(*[np.array([v], dtype=np.uint64) for v in c], k[0], k[1])]

    assert run([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert run([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert run([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0]) == \
        [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_keep_mask_rate_and_independence():
    m = keep_mask_ref(1 << 18, seed=123, site=7, p=0.1)
    assert abs(m.mean() - (1 - threshold16(0.1) / 65536)) < 0.003
    m2 = keep_mask_ref(1 << 18, seed=123, site=8, p=0.1)
    assert (m != m2).mean() > 0.1  # another site draws another mask
    assert np.array_equal(m, keep_mask_ref(1 << 18, seed=123, site=7, p=0.1))


def test_dropout_state_keys_advance_per_step():
    ds = DropoutState(0.1, "cpu", seed=5)
    k0 = ds.seed_host()
    ds.advance()
    assert ds.step == 1 and ds.seed_host() != k0 and ds.seed_host() == ds.key(1)
    ds.set_step(0)
    assert ds.seed_host() == k0


def _mask(st, site, numel):
    return torch.from_numpy(keep_mask_ref(numel, st.seed_host(), site, st.p))


@pytest.mark.gpu
def test_dropout_apply_and_embedding_kernels_match_oracle():
    from mtorus.ops import kernels as K

    st = DropoutState(0.1, "cuda", seed=3)
    x = torch.randn(256, 384, device="cuda").bfloat16()
    out = K.dropout_apply(x, st.args(41))
    m = _mask(st, 41, x.numel()).reshape(x.shape)
    want = torch.where(m, (x.float().cpu() * st.scale).bfloat16().float(), torch.zeros(1))
    assert torch.equal(out.float().cpu(), want)
    V, d, S = 100, 256, 64
    wte = torch.randn(V, d, device="cuda").bfloat16()
    wpe = torch.randn(S, d, device="cuda").bfloat16()
    ids = torch.randint(0, V, (4 * S,), device="cuda")
    e = K.embed_fwd(ids, wte, wpe, S, st.args(0xFFFF)).float().cpu()
    base = (wte[ids].float() + wpe[torch.arange(4 * S, device="cuda") % S].float()).bfloat16().float().cpu()
    m = _mask(st, 0xFFFF, 4 * S * d).reshape(4 * S, d)
    assert torch.allclose(e, torch.where(m, base * st.scale, torch.zeros(1)), rtol=1e-2, atol=1e-2)
    assert torch.equal(e == 0, ~m | (base == 0))


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [1, 2, 3])
def test_gemm_epilogue_dropout_modes(mode):
    from mtorus.ops import kernels as K

    st = DropoutState(0.1, "cuda", seed=9)
    M, N, Kd = 512, 512, 256
    g = torch.Generator(device="cuda").manual_seed(mode)
    a = (torch.randn(M, Kd, device="cuda", generator=g) * 0.1).bfloat16()
    b = (torch.randn(N, Kd, device="cuda", generator=g) * 0.1).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    res = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    site = 19
    m = _mask(st, site, M * N).reshape(M, N).cuda()
    y = a.float() @ b.float().t()
    if mode == 1:
        with K.gemm_dropout(st.args(site), 1):
            out = K.gemm(a, b, bias=bias, residual=res)
        want = res.float() + torch.where(m, (y + bias) * st.scale, torch.zeros(1, device="cuda"))
        assert ((out.float() - want).norm() / want.norm()).item() < 1e-2
    elif mode == 2:
        pre = torch.empty(M, N, device="cuda").bfloat16()
        act = torch.empty_like(pre)
        with K.gemm_dropout(st.args(site), 2):
            K.gemm(a, b, out=pre, bias=bias, act=act)
        want = torch.where(m, F.gelu(pre.float()) * st.scale, torch.zeros(1, device="cuda"))
        assert ((act.float() - want).norm() / want.norm()).item() < 1e-2
        assert torch.equal(act == 0, ~m | (want == 0))
    else:
        aux = torch.randn(M, N, device="cuda", generator=g).bfloat16()
        with K.gemm_dropout(st.args(site), 3):
            out = K.gemm(a, b, aux=aux)
        xg = aux.float().requires_grad_(True)
        F.gelu(xg).backward(torch.ones_like(xg))
        want = torch.where(m, y * st.scale, torch.zeros(1, device="cuda")) * xg.grad
        assert ((out.float() - want).norm() / want.norm()).item() < 1e-2
    # the setting applies to one launch only
    plain = K.gemm(a, b)
    assert ((plain.float() - y).norm() / y.norm()).item() < 1e-2


@pytest.mark.gpu
def test_attention_dropout_forward_and_backward_match_masked_reference():
    from mtorus.ops.attention import attention_bwd, attention_fwd, reference_attention

    B, S, H, dh = 2, 256, 2, 128
    st = DropoutState(0.1, "cuda", seed=21)
    site = 8 * 3
    g = torch.Generator(device="cuda").manual_seed(0)
    qkv = (torch.randn(B * S, 3 * H * dh, device="cuda", generator=g) * 0.5).bfloat16()
    keep = _mask(st, site, B * H * S * S).reshape(B, H, S, S).cuda()
    out, lse = attention_fwd(qkv, B, S, H, st.args(site))
    x = qkv.float().requires_grad_(True)
    ref = reference_attention(x, B, S, H, dh, keep=keep, p_drop=st.p)
    assert ((out.float() - ref).norm() / ref.norm()).item() < 2e-2
    dout = torch.randn(B * S, H * dh, device="cuda", generator=g).bfloat16()
    ref.backward(dout.float())
    dqkv = attention_bwd(dout, qkv, out, lse, B, S, H, drop=st.args(site))
    for i in range(3):  # dq, dk, dv
        got = dqkv[:, i * H * dh:(i + 1) * H * dh].float()
        want = x.grad[:, i * H * dh:(i + 1) * H * dh]
        assert ((got - want).norm() / want.norm()).item() < 3e-2, i


@pytest.mark.gpu
@pytest.mark.parametrize("recipe", ["tensor", "mx"])
def test_trainer_with_reference_dropout_trains_and_replays(recipe):
    """GptTrainer with the reference GPT's p = 0.1: trains on a repeated batch, the same
    seed gives the same losses, and the CUDA-graph replay draws fresh masks per step."""
    from mtorus.models.gpt import GptConfig
    from mtorus.training.engine import GptTrainer

    cfg = GptConfig(vocab_size=512, d_model=256, num_layers=2, num_heads=2, d_ff=1024, max_seq_len=256,
                    dropout=0.1)
    g = torch.Generator().manual_seed(3)
    t = torch.randint(0, 512, (2, 257), generator=g)
    ids, tgt = t[:, :-1].contiguous(), t[:, 1:].contiguous()
    curves = []
    for _ in range(2):
        tr = GptTrainer(cfg, device="cuda", lr=1e-3, init="normal", seed=0, fp8=True, fp8_recipe=recipe)
        assert tr.model.dropout_state is not None
        curves.append([tr.train_step(ids, tgt) for _ in range(6)])
    assert all(abs(a - b) <= 1e-5 * abs(b) for a, b in zip(curves[0], curves[1]))
    assert curves[0][-1] < curves[0][0]
    k0 = tr.model.dropout_state.seed_host()
    tr.capture(ids.cuda(), tgt.cuda())
    l1 = float(tr.graph_step(ids.cuda(), tgt.cuda()))
    k1 = tr.model.dropout_state.seed_host()
    assert k1 != k0 and l1 == l1
