"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""
import math
import os

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    from mtorus.ops import kernels

    return kernels


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.mark.parametrize("M,N,Kd", [(128, 256, 64), (256, 512, 128), (200, 136, 72), (1000, 1032, 520),
                                    (4096, 2048, 2048), (77, 8, 16)])
@pytest.mark.parametrize("layout", ["tn", "dgrad", "wgrad"])
def test_gemm_layouts(K, M, N, Kd, layout):
    torch.manual_seed(0)
    dev = "cuda"
    A = torch.randn(M, Kd, device=dev).bfloat16()
    B = torch.randn(N, Kd, device=dev).bfloat16()
    ref = A.float() @ B.float().t()
    if layout == "wgrad" and M % 8:
        pytest.skip("MN-major A needs M % 8 == 0 (16-byte TMA row stride)")
    if layout == "tn":
        out = K.gemm(A, B)
    elif layout == "dgrad":
        out = K.gemm(A, B.t().contiguous(), b_mn=True)
    else:
        out = K.gemm(A.t().contiguous(), B.t().contiguous(), a_mn=True, b_mn=True)
    torch.cuda.synchronize()
    assert K.gemm_status() == 0
    assert _rel(out, ref) < 1e-2, (layout, _rel(out, ref))


def test_gemm_epilogues(K):
    torch.manual_seed(1)
    M, N, Kd = 384, 520, 256
    A = torch.randn(M, Kd, device="cuda").bfloat16()
    B = torch.randn(N, Kd, device="cuda").bfloat16() * 0.1
    bias = torch.randn(N, device="cuda")
    res = torch.randn(M, N, device="cuda").bfloat16()
    base = A.float() @ B.float().t()
    # bias + residual
    out = K.gemm(A, B, bias=bias, residual=res)
    assert _rel(out, base + bias + res.float()) < 1e-2
    # gelu: out = pre, act = gelu(pre)
    act = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    pre = K.gemm(A, B, bias=bias, act=act)
    assert _rel(pre, base + bias) < 1e-2
    assert _rel(act, F.gelu(pre.float())) < 1e-2
    # dgelu via aux
    aux = torch.randn(M, N, device="cuda").bfloat16()
    x = aux.float().requires_grad_()
    F.gelu(x).backward(torch.ones_like(x))
    out = K.gemm(A, B, aux=aux)
    assert _rel(out, base * x.grad) < 1e-2
    # fp32 out, accumulate, alpha
    D = torch.randn(M, N, device="cuda")
    D0 = D.clone()
    alpha = torch.tensor([0.5], device="cuda")
    K.gemm(A, B, out=D, accumulate=True, alpha=alpha)
    assert _rel(D, D0 + 0.5 * base) < 1e-3
    torch.cuda.synchronize()
    assert K.gemm_status() == 0


@pytest.mark.parametrize("rows,d", [(1, 128), (37, 2048), (300, 1000), (64, 4096), (513, 768), (4099, 2048)])
def test_layernorm(K, rows, d):
    torch.manual_seed(2)
    x = torch.randn(rows, d, device="cuda").bfloat16()
    g = torch.randn(d, device="cuda")
    b = torch.randn(d, device="cuda")
    y, mean, rstd = K.layernorm_fwd(x, g, b, 1e-5)
    xr = x.float().requires_grad_()
    gr = g.clone().requires_grad_()
    br = b.clone().requires_grad_()
    yr = F.layer_norm(xr, (d,), gr, br, 1e-5)
    assert _rel(y, yr) < 1e-2
    dy = torch.randn(rows, d, device="cuda").bfloat16()
    yr.backward(dy.float())
    dg = torch.zeros(d, device="cuda")
    db = torch.zeros(d, device="cuda")
    dx = K.layernorm_bwd(dy, x, g, mean, rstd, dg, db, False)
    assert _rel(dx, xr.grad) < 2e-2
    assert _rel(dg, gr.grad) < 1e-2
    assert _rel(db, br.grad) < 1e-3
    # accumulate
    K.layernorm_bwd(dy, x, g, mean, rstd, dg, db, True)
    assert _rel(db, 2 * br.grad) < 1e-3
    if d % 256 == 0:
        # residual-branch gradient added inside the kernel
        dres = torch.randn(rows, d, device="cuda").bfloat16()
        dx2 = K.layernorm_bwd(dy, x, g, mean, rstd, dg, db, False, dres=dres)
        assert _rel(dx2, xr.grad + dres.float()) < 2e-2
        assert _rel(dg, gr.grad) < 1e-2


@pytest.mark.parametrize("T,V", [(4, 1000), (64, 50304), (7, 1003)])
def test_xent(K, T, V):
    torch.manual_seed(3)
    logits = (torch.randn(T, V, device="cuda") * 3).bfloat16()
    tgt = torch.randint(0, V, (T,), device="cuda")
    lf = logits.float().requires_grad_()
    ref = F.cross_entropy(lf, tgt)
    ref.backward()
    lg = logits.clone()
    rows = K.xent_fused(lg, tgt, None, 1.0 / T, True)
    assert abs(rows.mean().item() - ref.item()) < 1e-3 * max(1, abs(ref.item()))
    assert _rel(lg, lf.grad) < 2e-2


def test_embedding(K):
    torch.manual_seed(4)
    V, S, d, B = 500, 64, 256, 3
    wte = torch.randn(V, d, device="cuda").bfloat16()
    wpe = torch.randn(S, d, device="cuda").bfloat16()
    ids = torch.randint(0, V, (B, S), device="cuda")
    x = K.embed_fwd(ids.reshape(-1), wte, wpe, S)
    ref = (wte.float()[ids] + wpe.float()[None]).reshape(-1, d)
    assert _rel(x, ref) < 1e-2
    dy = torch.randn(B * S, d, device="cuda").bfloat16()
    dwte = torch.zeros(V, d, device="cuda")
    dwpe = torch.zeros(S, d, device="cuda")
    K.embed_bwd(ids.reshape(-1), dy, dwte, dwpe, S, False)
    rt = torch.zeros(V, d, device="cuda").index_add_(0, ids.reshape(-1), dy.float())
    assert _rel(dwte, rt) < 1e-4
    assert _rel(dwpe, dy.float().view(B, S, d).sum(0)) < 1e-4


def test_gelu_and_colsum(K):
    pre = torch.randn(33, 1024, device="cuda").bfloat16()
    bias = torch.randn(1024, device="cuda")
    p2 = pre.clone()
    act = K.bias_gelu_fwd(p2, bias)
    assert _rel(p2, pre.float() + bias) < 1e-2
    assert _rel(act, F.gelu(p2.float())) < 1e-2
    out = torch.zeros(1024, device="cuda")
    K.colsum_(pre, out, False)
    assert _rel(out, pre.float().sum(0)) < 1e-4
    big = torch.randn(5000, 2048, device="cuda").bfloat16()
    out = torch.ones(2048, device="cuda")
    K.colsum_(big, out, True, scale=torch.tensor([0.5], device="cuda"))
    assert _rel(out, 1 + 0.5 * big.float().sum(0)) < 1e-4


def test_adam_matches_reference(K):
    torch.manual_seed(5)
    n = 10007
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda") * 8.0  # gradients scaled by a loss scale of 8
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    w16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    st = torch.zeros(16, device="cuda")
    st[2] = 8.0
    pr, mr, vr = p.clone(), m.clone(), v.clone()
    for step in range(1, 4):
        K.grad_sumsq(g, st)
        K.optim_finalize(st, True, 2, 0.0, True)
        K.adam_step(p, m, v, g, w16, st, 1e-2, 0.9, 0.999, 1e-5, 0.0)
        # reference (scale is 8 for steps 1-2 then doubles after growth_interval=2)
        scale = 8.0 if step <= 2 else 16.0
        gu = g / scale
        mr = 0.9 * mr + 0.1 * gu
        vr = 0.999 * vr + 0.001 * gu * gu
        pr = pr - 1e-2 / (1 - 0.9 ** step) * mr / (vr.sqrt() / math.sqrt(1 - 0.999 ** step) + 1e-5)
    torch.cuda.synchronize()
    assert (p - pr).abs().max().item() < 1e-5
    assert _rel(w16, p) < 1e-2
    assert st[2].item() == 16.0  # scale doubled once after 2 clean steps


def test_overflow_skips_and_halves(K):
    p = torch.ones(64, device="cuda")
    g = torch.ones(64, device="cuda")
    g[3] = float("inf")
    m = torch.zeros(64, device="cuda")
    v = torch.zeros(64, device="cuda")
    st = torch.zeros(16, device="cuda")
    st[2] = 4.0
    K.grad_sumsq(g, st)
    K.optim_finalize(st, True, 100, 0.0, True)
    K.adam_step(p, m, v, g, None, st, 1e-2)
    torch.cuda.synchronize()
    assert torch.all(p == 1.0)
    assert st[2].item() == 2.0 and st[5].item() == 1.0


# ---------------------------------------------------------------- FP8
def _q(x, fmt, scale):
    dt = torch.float8_e4m3fn if fmt == 0 else torch.float8_e5m2
    mx = 448.0 if fmt == 0 else 57344.0
    return (x.float() * scale).clamp(-mx, mx).to(dt)


@pytest.mark.parametrize("fmt", [0, 1])
def test_fp8_quantize_matches_torch(fmt):
    from mtorus.ops import fp8 as F8

    x = (torch.randn(4099, 37, device="cuda") * 3).bfloat16()
    scale = torch.tensor([17.0], device="cuda")
    amax = torch.zeros(1, device="cuda")
    q = F8.quantize(x, fmt, scale, amax)
    ref = _q(x, fmt, 17.0).view(torch.uint8)
    assert torch.equal(q, ref)
    assert amax.item() == x.float().abs().max().item()


@pytest.mark.parametrize("layout", ["tn", "dgrad", "wgrad"])
@pytest.mark.parametrize("fa,fb", [(0, 0), (1, 0)])
def test_gemm_fp8(layout, fa, fb):
    from mtorus.ops import fp8 as F8

    torch.manual_seed(7)
    M, N, Kd = 512, 768, 384
    A = torch.randn(M, Kd, device="cuda")
    B = torch.randn(N, Kd, device="cuda")
    sa, sb = 20.0, 30.0
    A8, B8 = _q(A, fa, sa), _q(B, fb, sb)
    ref = (A8.float() / sa) @ (B8.float() / sb).t()
    ia = torch.tensor([1 / sa], device="cuda")
    ib = torch.tensor([1 / sb], device="cuda")
    if layout == "tn":
        out = F8.gemm_fp8(A8.view(torch.uint8), fa, B8.view(torch.uint8), fb, alpha=ia, alpha2=ib)
    elif layout == "dgrad":
        out = F8.gemm_fp8(A8.view(torch.uint8), fa, B8.t().contiguous().view(torch.uint8), fb, b_mn=True,
                          alpha=ia, alpha2=ib)
    else:
        out = F8.gemm_fp8(A8.t().contiguous().view(torch.uint8), fa, B8.t().contiguous().view(torch.uint8), fb,
                          a_mn=True, b_mn=True, alpha=ia, alpha2=ib, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert K_status() == 0
    assert _rel(out, ref) < 1e-2, _rel(out, ref)


def K_status():
    from mtorus.ops import kernels

    return kernels.gemm_status()


def test_fp8_state_delayed_scaling():
    from mtorus.ops import fp8 as F8

    st = F8.Fp8State("cuda", history=4)
    x = torch.randn(1024, device="cuda").bfloat16()
    q, inv = st.quantize(x, "a", F8.E4M3)
    amax = x.float().abs().max().item()
    assert abs(1.0 / inv.item() - 416.0 / amax) / (416.0 / amax) < 1e-6  # first step: current scaling
    st.end_step()
    q2, inv2 = st.quantize(x * 2, "a", F8.E4M3)
    assert abs(1.0 / inv2.item() - 416.0 / amax) / (416.0 / amax) < 1e-6  # delayed: previous amax
    st.end_step()
    q3, inv3 = st.quantize(x, "a", F8.E4M3)
    assert abs(1.0 / inv3.item() - 416.0 / (2 * amax)) / (416.0 / amax) < 1e-5


@pytest.mark.parametrize("B,S,H", [(1, 128, 1), (2, 256, 2), (1, 1024, 3)])
def test_attention_forward_backward(B, S, H):
    """tcgen05 flash attention (forward and backward) vs a plain fp32 PyTorch
    causal softmax attention."""
    from mtorus._ext import cuda as _cuda
    from mtorus.ops.attention import attention_bwd, attention_fwd, reference_attention

    torch.manual_seed(0)
    dh = 128
    qkv = (torch.randn(B * S, 3 * H * dh, device="cuda") * 1.5).bfloat16()
    out, lse = attention_fwd(qkv, B, S, H)
    torch.cuda.synchronize()
    assert _cuda().attn_status(True) == 0
    x = qkv.float().requires_grad_(True)
    ref = reference_attention(x, B, S, H, dh)
    assert _rel(out, ref) < 1e-2
    # log-sum-exp of the scaled scores
    q, k, _ = qkv.float().view(B, S, 3, H, dh).unbind(2)
    s = (q.transpose(1, 2) @ k.transpose(1, 2).transpose(-1, -2)) / dh ** 0.5
    s = s.masked_fill(torch.ones(S, S, dtype=torch.bool, device="cuda").triu(1), float("-inf"))
    assert torch.allclose(lse, torch.logsumexp(s, -1), atol=2e-2, rtol=1e-3)
    dout = torch.randn(B * S, H * dh, device="cuda").bfloat16()
    ref.backward(dout.float())
    dqkv = attention_bwd(dout, qkv, out, lse, B, S, H)
    torch.cuda.synchronize()
    assert _cuda().attn_status(True) == 0
    g = x.grad.view(B * S, 3, H * dh)
    d = dqkv.view(B * S, 3, H * dh)
    for i, name in enumerate("qkv"):
        assert _rel(d[:, i], g[:, i]) < 2e-2, (name, _rel(d[:, i], g[:, i]))


@pytest.mark.parametrize("rows,F", [(512, 256), (1000, 2048), (64, 8)])
@pytest.mark.parametrize("accumulate", [False, True])
def test_fp8_quantize_colsum(rows, F, accumulate):
    """Fused E5M2 quantisation + column sums == the separate quantise and fp32 column sums."""
    from mtorus.ops import fp8 as F8

    torch.manual_seed(0)
    x = (torch.randn(rows, F, device="cuda") * 3).bfloat16()
    st = F8.Fp8State("cuda", history=4, capacity=8)
    st.first_step = False
    s = st.slot("g", F8.E5M2)
    st.scale[s] = 100.0
    col = torch.full((F,), 0.5, device="cuda")
    q, _ = st.quantize_colsum(x, "g", F8.E5M2, col, accumulate)
    ref_q = F8.quantize(x, F8.E5M2, st.scale[s:s + 1])
    assert torch.equal(q, ref_q)
    ref_col = x.float().sum(0) + (0.5 if accumulate else 0.0)
    assert torch.allclose(col, ref_col, rtol=1e-4, atol=1e-3)
    assert abs(float(st.amax[s]) - float(x.float().abs().max())) < 1e-6


@pytest.mark.parametrize("rows,d", [(300, 256), (1024, 2048)])
def test_layernorm_fp8_output_matches_unfused(K, rows, d):
    """LayerNorm writing E4M3 codes == bf16 LayerNorm followed by the quantise kernel."""
    from mtorus.ops import fp8 as F8

    torch.manual_seed(0)
    x = (torch.randn(rows, d, device="cuda") * 2 + 0.5).bfloat16()
    gamma = torch.randn(d, device="cuda") * 0.2 + 1
    beta = torch.randn(d, device="cuda") * 0.1
    st = F8.Fp8State("cuda", history=4, capacity=8)
    st.first_step = False
    s = st.slot("h", F8.E4M3)
    st.scale[s] = 50.0
    q, _, mean, rstd = st.layernorm_quantize(x, gamma, beta, 1e-5, "h", F8.E4M3)
    h, mean_r, rstd_r = K.layernorm_fwd(x, gamma, beta, 1e-5)
    ref = F8.quantize(h, F8.E4M3, st.scale[s:s + 1])
    assert torch.equal(q, ref)
    assert torch.allclose(mean, mean_r) and torch.allclose(rstd, rstd_r)
    assert float(st.amax[s]) == float(h.float().abs().max())


@pytest.mark.parametrize("M,N,Kd", [(256, 512, 256), (1000, 1024, 512)])
def test_gemm_fp8_gelu_fp8_epilogue(M, N, Kd):
    """FP8 GEMM writing GELU(x W^T + b) as E4M3 codes == the bf16-GELU epilogue followed
    by the quantise kernel (codes and amax)."""
    from mtorus.ops import fp8 as F8

    torch.manual_seed(0)
    a = (torch.randn(M, Kd, device="cuda") * 0.5).to(torch.float8_e4m3fn).view(torch.uint8)
    b = (torch.randn(N, Kd, device="cuda") * 0.5).to(torch.float8_e4m3fn).view(torch.uint8)
    bias = torch.randn(N, device="cuda") * 0.1
    one = torch.full((1,), 0.05, device="cuda")
    pre_r = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    act_r = torch.empty_like(pre_r)
    F8.gemm_fp8(a, F8.E4M3, b, F8.E4M3, out=pre_r, bias=bias, act=act_r, alpha=one)
    scale = torch.full((1,), 20.0, device="cuda")
    amax = torch.zeros(1, device="cuda")
    pre = torch.empty_like(pre_r)
    a8 = torch.empty(M, N, dtype=torch.uint8, device="cuda")
    F8.gemm_fp8_gelu8(a, F8.E4M3, b, F8.E4M3, pre, a8, scale, amax, F8.E4M3, bias=bias, alpha=one)
    assert torch.equal(pre, pre_r)
    assert torch.equal(a8, F8.quantize(act_r, F8.E4M3, scale))
    assert float(amax) == float(act_r.float().abs().max())


def test_e5m2_encode_and_decode_mean_kernels_match_cpu_path():
    """One GPU: the E5M2 block encoder matches the PyTorch oracle byte for byte, and the
    fused decode-average (NCCL reducer path) matches the CPU path exactly."""
    from mtorus._ext import cuda as _cuda
    from mtorus.parallel.data_parallel import e5m2_decode, e5m2_encode

    g = torch.Generator().manual_seed(3)
    n, c = 3, 4096
    xs = [torch.randn(c, generator=g) * torch.logspace(-5, 3, c // 32).repeat_interleave(32) for _ in range(n)]
    xs[1][77] = float("inf")
    enc_cpu = [e5m2_encode(x) for x in xs]
    enc_gpu = [e5m2_encode(x.cuda()) for x in xs]
    for (cc, sc), (cg, sg) in zip(enc_cpu, enc_gpu):
        assert torch.equal(sc, sg.cpu())
        finite = sc != 255
        assert torch.equal(cc.view(-1, 32)[finite], cg.cpu().view(-1, 32)[finite])
    rc = torch.stack([e[0] for e in enc_cpu])
    rs = torch.stack([e[1] for e in enc_cpu])
    ref = (e5m2_decode(rc, rs).sum(0) * (1.0 / n)).to(torch.bfloat16)
    out = torch.empty(c, dtype=torch.bfloat16, device="cuda")
    _cuda().dp_decode_mean_e5m2(rc.cuda(), rs.cuda(), out)
    got = out.cpu()
    both_nan = torch.isnan(got.float()) & torch.isnan(ref.float())
    assert bool(both_nan[64:96].all())  # the block holding the Inf decodes to NaN
    assert torch.equal(got[~both_nan], ref[~both_nan])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fp8_wire_codec_kernels_match_reference(dtype):
    """The pipeline's FP8 wire encoder / decoder kernels agree with the PyTorch
    restatement byte for byte (ragged tail, zero block, NaN block included)."""
    from mtorus.pipeline import wire as W

    g = torch.Generator().manual_seed(5)
    x = (torch.randn(4133, generator=g) * torch.logspace(-6, 6, 4133)).to(dtype)
    x[96:128] = 0
    x[300] = float("nan")
    for fmt in (W.E4M3, W.E5M2):
        ref = W.encode_ref(x, fmt)
        got = W.encode(x.cuda(), fmt).cpu()
        n = x.numel()
        assert torch.equal(got[n:], ref[n:])  # every block's scale byte, the NaN block's 255 included
        keep = torch.ones(n, dtype=torch.bool)
        keep[288:320] = False  # the NaN block decodes to NaN whatever its codes
        assert torch.equal(got[:n][keep], ref[:n][keep])
        back = W.decode(got.cuda(), x.shape, dtype, fmt).cpu()
        want = W.decode_ref(ref, x.shape, dtype, fmt)
        assert torch.equal(torch.isnan(back), torch.isnan(want))
        ok = ~torch.isnan(want)
        assert torch.equal(back[ok], want[ok])


def test_xent_writes_e5m2_dlogits_like_the_separate_quantiser(K):
    """The cross-entropy kernel's E5M2 output: the codes the separate quantiser makes of the
    bf16 dlogits it would otherwise write, the same amax, the same loss; the logits are left
    untouched; and the column sums over the codes give the bias gradient of those codes."""
    from mtorus.ops import fp8 as F8

    T, V = 256, 50304
    g = torch.Generator(device="cuda").manual_seed(9)
    logits = (torch.randn(T, V, device="cuda", generator=g) * 3).bfloat16()
    tgt = torch.randint(0, V, (T,), device="cuda", generator=g)
    gs = torch.full((1,), 1024.0, device="cuda")
    scale = torch.full((1,), 4096.0, device="cuda")
    amax = torch.zeros(1, device="cuda")
    codes = torch.empty(T, V, dtype=torch.uint8, device="cuda")
    ref_logits = logits.clone()
    before = logits.clone()
    loss8 = K.xent_fused(logits, tgt, gs, 1.0 / T, True, out8=codes, out8_scale=scale, out8_amax=amax)
    assert torch.equal(logits, before)
    loss = K.xent_fused(ref_logits, tgt, gs, 1.0 / T, True)  # ref_logits now holds bf16 dlogits
    assert torch.equal(loss8, loss)
    amax_ref = torch.zeros(1, device="cuda")
    want = F8.quantize(ref_logits, F8.E5M2, scale, amax_ref)
    assert torch.equal(codes, want)
    assert torch.equal(amax, amax_ref)
    cs = torch.zeros(V, device="cuda")
    inv = 1.0 / scale
    K.colsum_e5m2_(codes, cs, False, scale=inv)
    dec = F8.dequantize(codes, inv, F8.E5M2)
    assert torch.allclose(cs, dec.sum(0), rtol=1e-5, atol=1e-6)


def test_gemm_epilogue_gelu_matches_fp32_erf_gelu(K):
    """The CTA-pair GEMM epilogue's GELU (alternating the special-function-unit and the
    FMA-pipe forms over its values) and its dGELU agree with PyTorch's fp32 erf GELU
    to bf16 rounding: D = X . I reproduces X exactly, so act = GELU(X); with A = 1 and
    aux = X the dGELU epilogue yields GELU'(X)."""
    M = N = 256
    x = (torch.rand(M, N, device="cuda") * 16 - 8).bfloat16()
    eye = torch.eye(N, device="cuda").bfloat16()
    pre = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    act = torch.empty_like(pre)
    K.gemm(x, eye, out=pre, act=act)
    assert torch.equal(pre, x)
    ref = F.gelu(x.float())
    assert bool(((act.float() - ref).abs() <= 2.0 ** -8 * ref.abs() + 2e-6).all())
    xg = x.float().requires_grad_(True)
    F.gelu(xg).backward(torch.ones_like(xg))
    ones = torch.zeros(M, N, device="cuda").bfloat16()
    ones[:, 0] = 1.0
    e0 = torch.zeros(N, N, device="cuda").bfloat16()
    e0[:, 0] = 1.0  # D[m, n] = sum_k ones[m, k] e0[n, k] = 1
    d = K.gemm(ones, e0, aux=x)
    assert bool(((d.float() - xg.grad).abs() <= 2.0 ** -8 * xg.grad.abs() + 2e-6).all())


def test_gelu_kernels_match_fp32_erf_gelu_elementwise(K):
    """The epilogues' GELU / GELU' (erf from Abramowitz & Stegun 7.1.26, |error| <=
    1.5e-7) agree with PyTorch's fp32 erf GELU to bf16 rounding, element by element,
    over [-8, 8] (both tails included)."""
    x = torch.linspace(-8, 8, 4096 * 8, device="cuda").reshape(-1, 4096).bfloat16()
    ref = F.gelu(x.float())
    act = K.bias_gelu_fwd(x.clone(), None)
    assert bool(((act.float() - ref).abs() <= 2.0 ** -8 * ref.abs() + 2e-6).all())
    xg = x.float().requires_grad_(True)
    F.gelu(xg).backward(torch.ones_like(xg))
    d = torch.ones_like(x)
    K.gelu_bwd_(d, x)
    assert bool(((d.float() - xg.grad).abs() <= 2.0 ** -8 * xg.grad.abs() + 2e-6).all())
