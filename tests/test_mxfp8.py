"""MXFP8 block-scaled quantisation (1x32 blocks, UE8M0 scales) and the tcgen05
block-scaled GEMM.

CPU tests pin the reference quantiser: the block-exponent rule, the round trip,
special blocks and the tensor-memory atom layout of the scales.  The GPU tests
compare the CUDA quantiser with the reference byte for byte and the GEMM with an
fp32 product of the dequantised operands (and with cuBLAS's MX GEMM).
"""
import pytest
import torch

import mtorus.ops.mxfp8 as mxfp8_mod

from mtorus.ops.mxfp8 import (E4M3, E5M2, MX_FMT_MAX, MxTensor, gemm_mxfp8, gemm_mxfp8_mx_out, gemm_mxfp8_ref,
                              mx_dequantize, mx_linear, mx_quantize, mx_quantize_rc, mx_quantize_ref, sf_numel,
                              sf_offsets)


def _blocky(R, K, seed=0):
    """Rows whose 32-blocks span many magnitudes (2^-20 .. 2^20)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(R, K // 32, 32, generator=g)
    mag = torch.ldexp(torch.ones(R, K // 32, 1), torch.randint(-20, 21, (R, K // 32, 1), generator=g).float())
    return (x * mag).reshape(R, K)


def test_sf_layout_is_a_permutation_of_the_valid_slots():
    R, K = 300, 544  # partial row block and partial K atom
    off = sf_offsets(R, K).reshape(-1)
    assert off.unique().numel() == off.numel()
    assert int(off.min()) >= 0 and int(off.max()) < sf_numel(R, K)
    assert sf_numel(R, K) == 3 * 5 * 512
    # row r, block j of atom (0, 0): (r % 32) * 16 + (r // 32) * 4 + j
    assert int(sf_offsets(128, 128)[37, 2]) == 5 * 16 + 1 * 4 + 2
    # next K atom of the same row block, then the next row block
    assert int(sf_offsets(256, 256)[0, 4]) == 512
    assert int(sf_offsets(256, 256)[128, 0]) == 2 * 512


@pytest.mark.parametrize("fmt", [E4M3, E5M2])
def test_block_exponent_rule_and_round_trip(fmt):
    R, K = 160, 256
    x = _blocky(R, K, seed=fmt)
    t = mx_quantize_ref(x, fmt)
    fmax = MX_FMT_MAX[fmt]
    byte = t.sf[sf_offsets(R, K)].long()
    X = byte - 127
    amax = x.reshape(R, K // 32, 32).abs().amax(-1).double()
    scaled_max = amax * torch.pow(2.0, -X.double())
    # smallest X with amax <= fmax * 2^X: amax * 2^-X lies in (fmax / 2, fmax]
    assert bool((scaled_max <= fmax).all()) and bool((scaled_max > fmax / 2).all())
    y = mx_dequantize(t)
    rel = 2.0 ** -4 if fmt == E4M3 else 2.0 ** -3  # half an ulp of a 3 / 2-bit mantissa
    sub = (2.0 ** -9 if fmt == E4M3 else 2.0 ** -16) * torch.pow(2.0, X.double())  # subnormal spacing / 2
    bound = rel * x.abs().double() + sub.repeat_interleave(32, dim=1)
    assert bool(((y.double() - x.double()).abs() <= bound).all())


def test_padding_zero_and_nonfinite_blocks():
    R, K = 130, 96  # 2 row blocks (second mostly padding), 3 of the 4 K-blocks of the atom
    x = torch.randn(R, K)
    x[3, 32:64] = 0.0
    x[5, 7] = float("nan")
    x[6, 70] = float("inf")
    t = mx_quantize_ref(x, E4M3)
    off = sf_offsets(R, K)
    assert int(t.sf[off[3, 1]]) == 127
    assert int(t.codes[3, 32:64].count_nonzero()) == 0
    assert int(t.sf[off[5, 0]]) == 255 and int(t.sf[off[6, 2]]) == 255
    used = torch.zeros(sf_numel(R, K), dtype=torch.bool)
    used[off.reshape(-1)] = True
    assert bool((t.sf[~used] == 127).all())
    y = mx_dequantize(t)
    assert bool(torch.isnan(y[5, :32]).all()) and bool(torch.isfinite(y[4]).all())


def test_cpu_entry_point_uses_the_reference():
    x = _blocky(64, 128, seed=3)
    a, b = mx_quantize(x, E4M3), mx_quantize_ref(x, E4M3)
    assert torch.equal(a.codes, b.codes) and torch.equal(a.sf, b.sf)


def test_reference_gemm_matches_fp32_product_of_dequantised_operands():
    a = mx_quantize_ref(_blocky(64, 96, seed=4) * 1e-3, E4M3)
    b = mx_quantize_ref(_blocky(48, 96, seed=5) * 1e-3, E4M3)
    da, db = mx_dequantize(a).double(), mx_dequantize(b).double()
    ref = da @ db.t()
    mag = da.abs() @ db.abs().t()  # fp32 summation error is relative to this, not to |ref|
    assert bool(((gemm_mxfp8_ref(a, b).double() - ref).abs() <= 1e-5 * mag).all())


def test_mx_linear_cpu_oracle_gradients():
    """All three GEMMs of the MXFP8 linear: forward on row-wise x / W, dgrad on row-wise
    dY with column-wise W, wgrad on column-wise dY and x (E5M2 gradients)."""
    torch.manual_seed(0)
    T, I, O = 64, 96, 128
    x = (torch.randn(T, I) * 0.5).bfloat16().float().requires_grad_(True)
    w = (torch.randn(O, I) * 0.05).requires_grad_(True)
    b = torch.randn(O, requires_grad=True)
    y = mx_linear(x, w, b)
    dy = torch.randn(T, O) * 1e-2
    y.backward(dy.bfloat16().float())
    xr, xc = mx_quantize_rc(x.detach().bfloat16(), E4M3)
    wr, wc = mx_quantize_rc(w.detach().bfloat16(), E4M3)
    dyr, dyc = mx_quantize_rc(dy.bfloat16(), E5M2)
    assert torch.equal(y.detach(), (mx_dequantize(xr) @ mx_dequantize(wr).t() + b.detach()).bfloat16())
    assert torch.equal(x.grad, (mx_dequantize(dyr) @ mx_dequantize(wc).t()).bfloat16().float())
    assert torch.allclose(w.grad, mx_dequantize(dyc) @ mx_dequantize(xc).t(), rtol=1e-6, atol=1e-9)
    assert torch.allclose(b.grad, dy.bfloat16().float().sum(0), rtol=1e-6, atol=1e-6)
    # and close to the unquantised layer (E4M3 / E5M2 with per-32 scales: a few percent)
    ref_y = x.detach() @ w.detach().t() + b.detach()
    assert float((y.detach().float() - ref_y).norm() / ref_y.norm()) < 0.05
    ref_dw = dy.t() @ x.detach()
    assert float((w.grad - ref_dw).norm() / ref_dw.norm()) < 0.1


def test_mx_quantize_rc_cpu_is_row_and_transposed_reference():
    x = _blocky(96, 64, seed=9)
    r, c = mx_quantize_rc(x, E4M3)
    assert torch.equal(r.codes, mx_quantize_ref(x, E4M3).codes)
    assert torch.equal(c.codes, mx_quantize_ref(x.t().contiguous(), E4M3).codes)
    assert torch.equal(c.sf, mx_quantize_ref(x.t().contiguous(), E4M3).sf)


# ---------------------------------------------------------------- GPU


def test_mx_quantize_rc_cpu_activation_modes():
    """act="gelu" / "dgelu" on the CPU: the quantiser of bf16(GELU(x)) / bf16(x * GELU'(aux))
    with the erf GELU."""
    g = torch.Generator().manual_seed(3)
    pre = (torch.randn(64, 96, generator=g) * 2).to(torch.bfloat16)
    dact = (torch.randn(64, 96, generator=g) * 1e-2).to(torch.bfloat16)
    r, c = mx_quantize_rc(pre, E4M3, act="gelu")
    x = pre.float()
    want = (0.5 * x * (1.0 + torch.erf(x * 0.7071067811865476))).to(torch.bfloat16)
    assert torch.equal(r.codes, mx_quantize_ref(want, E4M3).codes)
    assert torch.equal(c.codes, mx_quantize_ref(want.t(), E4M3).codes)
    cs = torch.zeros(96)
    r, c = mx_quantize_rc(dact, E5M2, colsum=cs, accumulate=False, act="dgelu", aux=pre)
    d = dact.float() * (0.5 * (1.0 + torch.erf(x * 0.7071067811865476)) + x * torch.exp(-0.5 * x * x) * 0.3989422804014327)
    d = d.to(torch.bfloat16)
    assert torch.equal(r.codes, mx_quantize_ref(d, E5M2).codes)
    assert torch.allclose(cs, d.float().sum(0))
    with pytest.raises(ValueError):
        mx_quantize_rc(dact, E5M2, act="dgelu")


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", [E4M3, E5M2])
def test_cuda_quantiser_matches_reference(fmt):
    x = _blocky(300, 544, seed=7).to(torch.bfloat16)
    x[11, 40] = float("nan")
    ref = mx_quantize_ref(x.float(), fmt)
    got = mx_quantize(x.cuda(), fmt)
    assert torch.equal(got.sf.cpu(), ref.sf)
    finite_rows = torch.isfinite(x.float()).all(1)
    assert torch.equal(got.codes.cpu()[finite_rows], ref.codes[finite_rows])


@pytest.mark.gpu
@pytest.mark.parametrize("shape,fmts", [((512, 512, 512), (E4M3, E4M3)), ((300, 264, 544), (E4M3, E4M3)),
                                        ((256, 2048, 1024), (E5M2, E4M3))])
def test_block_scaled_gemm_matches_fp32_oracle(shape, fmts):
    M, N, K = shape
    g = torch.Generator().manual_seed(M + N + K)
    xa = (_blocky(M, K, seed=1) * 1e-4).to(torch.bfloat16)
    xb = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    a, b = mx_quantize(xa.cuda(), fmts[0]), mx_quantize(xb.cuda(), fmts[1])
    ref = gemm_mxfp8_ref(MxTensor(a.codes.cpu(), a.sf.cpu(), a.fmt), MxTensor(b.codes.cpu(), b.sf.cpu(), b.fmt))
    da = mx_dequantize(MxTensor(a.codes.cpu(), a.sf.cpu(), a.fmt)).double()
    db = mx_dequantize(MxTensor(b.codes.cpu(), b.sf.cpu(), b.fmt)).double()
    mag = (da.abs() @ db.abs().t()).float()
    out = gemm_mxfp8(a, b, out_dtype=torch.float32, impl="own")
    torch.cuda.synchronize()
    err = (out.cpu() - ref).abs()
    assert bool((err <= 1e-5 * mag + 1e-30).all()), float((err / mag.clamp_min(1e-30)).max())
    out16 = gemm_mxfp8(a, b, impl="own").float().cpu()
    assert bool(((out16 - ref).abs() <= 1e-2 * ref.abs() + 1e-5 * mag + 1e-30).all())


@pytest.mark.gpu
def test_block_scaled_gemm_both_operands_blocky():
    """Block exponents spread over 2^-20..2^20 in A and B: every B row's scales (the
    CTA pair's 256 rows live in two scale atoms per CTA) must reach the right rows."""
    M, N, K = 512, 768, 512
    xa = (_blocky(M, K, seed=11) * 1e-4).to(torch.bfloat16)
    xb = (_blocky(N, K, seed=12) * 1e-4).to(torch.bfloat16)
    a, b = mx_quantize(xa.cuda(), E4M3), mx_quantize(xb.cuda(), E4M3)
    ref = gemm_mxfp8_ref(MxTensor(a.codes.cpu(), a.sf.cpu(), a.fmt), MxTensor(b.codes.cpu(), b.sf.cpu(), b.fmt))
    da = mx_dequantize(MxTensor(a.codes.cpu(), a.sf.cpu(), a.fmt)).double()
    db = mx_dequantize(MxTensor(b.codes.cpu(), b.sf.cpu(), b.fmt)).double()
    mag = (da.abs() @ db.abs().t()).float()
    out = gemm_mxfp8(a, b, out_dtype=torch.float32, impl="own")
    err = (out.cpu() - ref).abs()
    assert bool((err <= 1e-5 * mag + 1e-30).all()), float((err / mag.clamp_min(1e-30)).max())


@pytest.mark.gpu
def test_block_scaled_gemm_agrees_with_cublas_mx():
    """cuBLAS MX GEMM (torch._scaled_mm with e8m0 scales) reads the same scale layout."""
    M, N, K = 512, 768, 1024
    a = mx_quantize((torch.randn(M, K) * 3).to(torch.bfloat16).cuda())
    b = mx_quantize((torch.randn(N, K) * 0.02).to(torch.bfloat16).cuda())
    try:
        lib = torch._scaled_mm(a.codes.view(torch.float8_e4m3fn), b.codes.view(torch.float8_e4m3fn).t(),
                               a.sf.view(torch.float8_e8m0fnu).reshape(M, -1),
                               b.sf.view(torch.float8_e8m0fnu).reshape(N, -1), out_dtype=torch.float32)
    except (RuntimeError, AttributeError, TypeError) as e:
        pytest.skip(f"torch._scaled_mm has no MX path here: {e}")
    out = gemm_mxfp8(a, b, out_dtype=torch.float32, impl="own")
    assert torch.allclose(out, lib, rtol=1e-4, atol=1e-4 * float(lib.abs().max()))


@pytest.mark.gpu
@pytest.mark.parametrize("out_dtype,bias", [(torch.float32, False), (torch.bfloat16, True)])
def test_library_path_matches_own_kernel(out_dtype, bias):
    """The plain-GEMM routing to cuBLASLt (E5M2 x E4M3 as in dgrad / wgrad, a bias as in the
    QKV projection) gives what gemm_2sm_kernel gives, and "auto" takes it."""
    M, N, K = 512, 768, 1024
    a = mx_quantize((_blocky(M, K, seed=21) * 1e-3).to(torch.bfloat16).cuda(), E5M2)
    b = mx_quantize((torch.randn(N, K) * 0.02).to(torch.bfloat16).cuda(), E4M3)
    bb = (torch.randn(N) * 0.1).to(torch.bfloat16).float().cuda() if bias else None
    own = gemm_mxfp8(a, b, out_dtype=out_dtype, bias=bb, impl="own").float()
    lib = gemm_mxfp8(a, b, out_dtype=out_dtype, bias=bb, impl="library").float()
    auto = gemm_mxfp8(a, b, out_dtype=out_dtype, bias=bb).float()
    tol = 1e-5 if out_dtype == torch.float32 else 8e-3
    assert ((lib - own).norm() / own.norm()).item() < tol
    if mxfp8_mod.LIBRARY_PLAIN_GEMM:
        assert torch.equal(auto, lib)
    with pytest.raises(ValueError):
        gemm_mxfp8(a, b, out_dtype=torch.float32, accumulate=True, impl="library")


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(256, 512), (96, 320)])
def test_cuda_row_col_quantiser_matches_reference(shape):
    R, C = shape
    x = _blocky(R, C, seed=R).to(torch.bfloat16)
    cs = torch.full((C,), 5.0, device="cuda")
    r, c = mx_quantize_rc(x.cuda(), E4M3, colsum=cs, accumulate=True)
    rr, cr = mx_quantize_ref(x.float(), E4M3), mx_quantize_ref(x.float().t().contiguous(), E4M3)
    assert torch.equal(r.codes.cpu(), rr.codes) and torch.equal(r.sf.cpu(), rr.sf)
    assert torch.equal(c.codes.cpu(), cr.codes) and torch.equal(c.sf.cpu(), cr.sf)
    # the bias-gradient column sums of the same pass (fp32, added to the buffer)
    want = x.double().sum(0) + 5.0
    assert torch.allclose(cs.cpu().double(), want, rtol=1e-5, atol=1e-5 * float(x.double().abs().sum(0).max()))


@pytest.mark.gpu
@pytest.mark.parametrize("M,N", [(512, 768), (384, 384)])
def test_gemm_epilogue_mx_output_matches_unfused_quantiser(M, N):
    """The GEMM epilogue that quantises its own output (row and column MXFP8 codes,
    both scale atoms, column sums) writes exactly what the separate quantiser makes
    of the bf16 tensor the unfused epilogue would store: GELU of the FFN1
    pre-activation (E4M3) and the dGELU'd FFN2 dgrad (E5M2).  M = 384 leaves the
    second CTA of the last pair entirely past M."""
    K = 256
    g = torch.Generator().manual_seed(M + N)
    a = mx_quantize((torch.randn(M, K, generator=g) * 0.5).to(torch.bfloat16).cuda())
    b = mx_quantize((torch.randn(N, K, generator=g) * 0.1).to(torch.bfloat16).cuda())
    bias = (torch.randn(N, generator=g) * 0.1).cuda()
    # FFN1: pre-activation stored, GELU quantised
    pre_ref = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    act_ref = torch.empty_like(pre_ref)
    gemm_mxfp8(a, b, out=pre_ref, bias=bias, act=act_ref)
    r_ref, c_ref = mx_quantize_rc(act_ref, E4M3)
    pre = torch.empty_like(pre_ref)
    d, r, c = gemm_mxfp8_mx_out(a, b, E4M3, out=pre, bias=bias, gelu=True)
    torch.cuda.synchronize()
    assert torch.equal(d, pre_ref)
    for got, want in ((r, r_ref), (c, c_ref)):
        assert torch.equal(got.codes, want.codes) and torch.equal(got.sf, want.sf)
    # FFN2 dgrad: dGELU with the pre-activation as aux, E5M2 codes, bias-gradient sums, no bf16 store
    gd = mx_quantize((torch.randn(M, K, generator=g) * 1e-3).to(torch.bfloat16).cuda(), E5M2)
    dpre_ref = gemm_mxfp8(gd, b, aux=pre_ref)
    cs_ref = torch.full((N,), 0.5, device="cuda")
    r_ref, c_ref = mx_quantize_rc(dpre_ref, E5M2, colsum=cs_ref, accumulate=True)
    cs = torch.full((N,), 0.5, device="cuda")
    d, r, c = gemm_mxfp8_mx_out(gd, b, E5M2, aux=pre_ref, colsum=cs, accumulate=True, store_d=False)
    torch.cuda.synchronize()
    assert d is None
    for got, want in ((r, r_ref), (c, c_ref)):
        assert torch.equal(got.codes, want.codes) and torch.equal(got.sf, want.sf)
    assert torch.allclose(cs, cs_ref, rtol=1e-5, atol=1e-5 * float(dpre_ref.float().abs().sum(0).max()))


@pytest.mark.gpu
def test_long_k_residual_gemm_library_route_matches_own_kernel():
    """A residual GEMM with K >= LIBRARY_RESIDUAL_MIN_K (the FFN2 forward) runs as the library GEMM
    plus a bf16 add under "auto"; it agrees with the own kernel's fused residual epilogue to bf16
    rounding."""
    M, N, K = 256, 512, mxfp8_mod.LIBRARY_RESIDUAL_MIN_K
    a = mx_quantize((torch.randn(M, K) * 0.5).to(torch.bfloat16).cuda())
    b = mx_quantize((torch.randn(N, K) * 0.02).to(torch.bfloat16).cuda())
    bias = (torch.randn(N) * 0.1).to(torch.bfloat16).float().cuda()
    res = (torch.randn(M, N) * 2).to(torch.bfloat16).cuda()
    own = gemm_mxfp8(a, b, bias=bias, residual=res, impl="own").float()
    auto = gemm_mxfp8(a, b, bias=bias, residual=res).float()
    assert ((auto - own).norm() / own.norm()).item() < 8e-3
    assert ((auto - own).abs() <= 2e-2 * own.abs() + 1e-2).all()


@pytest.mark.gpu
@pytest.mark.parametrize("R,C", [(512, 768), (96, 320)])
def test_row_col_quantiser_gelu_and_dgelu_match_elementwise_then_quantise(R, C):
    """The quantiser's GELU / dGELU source modes (the FFN1 output and the FFN2 dgrad after a
    library GEMM) give exactly what the elementwise GELU / dGELU kernels followed by the
    plain quantiser give: the same bf16 values, codes, scale atoms and column sums."""
    from mtorus.ops import kernels as K

    g = torch.Generator().manual_seed(R + C)
    pre = (torch.randn(R, C, generator=g) * 2.0).to(torch.bfloat16).cuda()
    r, c = mx_quantize_rc(pre, E4M3, act="gelu")
    r_ref, c_ref = mx_quantize_rc(K.bias_gelu_fwd(pre), E4M3)
    for got, want in ((r, r_ref), (c, c_ref)):
        assert torch.equal(got.codes, want.codes) and torch.equal(got.sf, want.sf)
    dact = (torch.randn(R, C, generator=g) * 1e-3).to(torch.bfloat16).cuda()
    cs = torch.full((C,), 0.25, device="cuda")
    r, c = mx_quantize_rc(dact, E5M2, colsum=cs, accumulate=True, act="dgelu", aux=pre)
    dpre = dact.clone()
    K.gelu_bwd_(dpre, pre)
    cs_ref = torch.full((C,), 0.25, device="cuda")
    r_ref, c_ref = mx_quantize_rc(dpre, E5M2, colsum=cs_ref, accumulate=True)
    torch.cuda.synchronize()
    for got, want in ((r, r_ref), (c, c_ref)):
        assert torch.equal(got.codes, want.codes) and torch.equal(got.sf, want.sf)
    assert torch.allclose(cs, cs_ref, rtol=1e-5, atol=1e-5 * float(dpre.float().abs().sum(0).max()))


@pytest.mark.gpu
def test_attention_epilogue_mx_output_matches_quantiser():
    """The attention forward's MX-output epilogue writes exactly what the row / column
    quantiser makes of the bf16 output it stores (codes and both scale atoms)."""
    from mtorus.ops.attention import attention_fwd

    B, S, H = 2, 256, 2
    g = torch.Generator().manual_seed(5)
    qkv = (torch.randn(B * S, 3 * H * 128, generator=g) * 0.5).to(torch.bfloat16).cuda()
    out, lse, rows, cols = attention_fwd(qkv, B, S, H, mx_fmt=E4M3)
    plain, _ = attention_fwd(qkv, B, S, H)
    assert torch.equal(out, plain)
    r_ref, c_ref = mx_quantize_rc(out, E4M3)
    for got, want in ((rows, r_ref), (cols, c_ref)):
        assert torch.equal(got.codes, want.codes) and torch.equal(got.sf, want.sf)


@pytest.mark.gpu
def test_row_col_quantiser_reads_leading_columns_from_fp32():
    """xq: the first 128 columns come from an fp32 matrix (rounded to bf16 on load), the
    rest from the bf16 tensor -- the attention backward's fp32 dQ beside its bf16 dK / dV."""
    R, C = 256, 384
    x = _blocky(R, C, seed=3).to(torch.bfloat16)
    xq = _blocky(R, 128, seed=4).float() * 1.37
    x_nan = x.clone()
    x_nan[:, :128] = float("nan")  # must not be read
    cs = torch.zeros(C, device="cuda")
    r, c = mx_quantize_rc(x_nan.cuda(), E5M2, colsum=cs, xq=xq.cuda())
    full = x.clone()
    full[:, :128] = xq.to(torch.bfloat16)
    rr, cr = mx_quantize_ref(full.float(), E5M2), mx_quantize_ref(full.float().t().contiguous(), E5M2)
    assert torch.equal(r.codes.cpu(), rr.codes) and torch.equal(r.sf.cpu(), rr.sf)
    assert torch.equal(c.codes.cpu(), cr.codes) and torch.equal(c.sf.cpu(), cr.sf)
    assert torch.allclose(cs.cpu().double(), full.double().sum(0), rtol=1e-5,
                          atol=1e-5 * float(full.double().abs().sum(0).max()))


@pytest.mark.gpu
def test_mx_linear_cuda_matches_cpu_oracle():
    torch.manual_seed(1)
    T, I, O = 512, 256, 768
    x = (torch.randn(T, I) * 0.5).bfloat16()
    w = torch.randn(O, I) * 0.05
    b = torch.randn(O)
    dy = (torch.randn(T, O) * 1e-2).bfloat16()
    outs = {}
    for dev in ("cpu", "cuda"):
        xv = x.float().clone().to(dev).requires_grad_(True)
        wv = w.clone().to(dev).requires_grad_(True)
        bv = b.clone().to(dev).requires_grad_(True)
        y = mx_linear(xv, wv, bv)
        y.backward(dy.float().to(dev))
        outs[dev] = [t.detach().float().cpu() for t in (y, xv.grad, wv.grad, bv.grad)]
    for g, r in zip(outs["cuda"], outs["cpu"]):
        assert torch.allclose(g, r, rtol=2e-2, atol=1e-3 * float(r.abs().max()))


def test_gpt_trains_with_mx_linears_on_cpu():
    """The reference GPT with every Linear on the MXFP8 recipe (CPU oracle) follows the
    fp32 model's loss curve within a few percent."""
    from mtorus.models.gpt import GptConfig, GptModel
    from mtorus.ops.mxfp8 import enable_mx_linears

    cfg = GptConfig(256, 64, 2, 2, 256, 32, 0.0)
    losses = {}
    for mx in (False, True):
        torch.manual_seed(0)
        m = GptModel(cfg, init="normal")
        if mx:
            assert enable_mx_linears(m) == 2 * 4 + 2 * 2 + 1  # q/k/v/out, ffn in/out per block, lm head
        opt = torch.optim.Adam(m.parameters(), lr=3e-3)
        g = torch.Generator().manual_seed(1)
        data = torch.randint(0, 256, (8, 33), generator=g)
        curve = []
        for _ in range(6):
            logits = m(data[:, :-1])
            loss = torch.nn.functional.cross_entropy(logits.reshape(-1, 256).float(), data[:, 1:].reshape(-1))
            opt.zero_grad()
            loss.backward()
            opt.step()
            curve.append(float(loss.detach()))
        losses[mx] = curve
    assert losses[True][-1] < losses[True][0]
    for a, b in zip(losses[True], losses[False]):
        assert abs(a - b) / b < 0.05


@pytest.mark.gpu
def test_fused_trainer_mx_recipe_tracks_tensor_recipe():
    """GptTrainer with the MXFP8 recipe (block-scaled forward, dgrad and wgrad in the
    fused blocks) trains like the per-tensor FP8 recipe on a small model.  The data is
    two fixed batches seen in turn, so that the loss has something to learn (uniform
    random tokens have nothing below ln V)."""
    from mtorus.models.gpt import GptConfig
    from mtorus.training.engine import GptTrainer

    cfg = GptConfig(vocab_size=512, d_model=256, num_layers=2, num_heads=2, d_ff=1024, max_seq_len=128, dropout=0.0)
    g = torch.Generator().manual_seed(3)
    fixed = [torch.randint(0, 512, (4, 129), generator=g) for _ in range(2)]
    data = [fixed[i % 2] for i in range(12)]
    curves = {}
    for recipe in ("tensor", "mx"):
        tr = GptTrainer(cfg, device="cuda", lr=1e-3, init="normal", seed=0, fp8=True, fp8_recipe=recipe)
        curve = []
        for t in data:
            curve.append(float(tr.train_step(t[:, :-1].contiguous(), t[:, 1:].contiguous())))
        curves[recipe] = curve
    assert curves["mx"][-1] < curves["mx"][0]
    for a, b in zip(curves["mx"], curves["tensor"]):
        assert abs(a - b) / b < 0.05


def test_mx_layernorm_reference_path():
    from mtorus.ops.mxfp8 import mx_layernorm_rc

    torch.manual_seed(4)
    x = (torch.randn(64, 256) * 3 + 1).bfloat16()
    g, b = torch.rand(256) + 0.5, torch.randn(256) * 0.1
    r, c, mean, rstd = mx_layernorm_rc(x, g, b, 1e-5)
    h = torch.nn.functional.layer_norm(x.float(), (256,), g, b, 1e-5)
    assert torch.allclose(mean, x.float().mean(-1), atol=1e-5)
    assert float((mx_dequantize(r) - h).abs().max()) <= 2 ** -4 * float(h.abs().max()) + 1e-6
    hb = ((x.float() - mean[:, None]) * rstd[:, None] * g + b).bfloat16().float()
    assert torch.equal(c.codes, mx_quantize_ref(hb.t().contiguous(), E4M3).codes)


@pytest.mark.gpu
def test_cuda_layernorm_mx_matches_reference():
    from mtorus.ops.mxfp8 import mx_layernorm_rc

    torch.manual_seed(5)
    R, d = 256, 2048
    x = (torch.randn(R, d) * 2 + 0.5).bfloat16()
    g, b = torch.rand(d) + 0.5, torch.randn(d) * 0.1
    r_ref, c_ref, m_ref, s_ref = mx_layernorm_rc(x, g, b, 1e-5)
    r, c, m, s = mx_layernorm_rc(x.cuda(), g.cuda(), b.cuda(), 1e-5)
    assert torch.allclose(m.cpu(), m_ref, atol=1e-4) and torch.allclose(s.cpu(), s_ref, rtol=1e-4)
    # bf16 rounding of the normalised value may differ by one ulp: compare the decoded operands
    for got, ref in ((r, r_ref), (c, c_ref)):
        dg = mx_dequantize(MxTensor(got.codes.cpu(), got.sf.cpu(), got.fmt))
        dr = mx_dequantize(ref)
        assert float((dg - dr).abs().max()) <= 2 ** -3 * float(dr.abs().max())
        assert float((got.sf.cpu() == ref.sf).float().mean()) > 0.99


def test_reserved_sms_reach_the_library_gemms(monkeypatch):
    """set_reserved_sms keeps the reduce-scatter's SMs out of both GEMM families: the own
    kernels' grid size and torch's cuBLASLt SM carveout; 0 releases both, and the switch
    leaves the library alone."""
    from mtorus.ops import kernels as K

    seen = []

    class FakeExt:
        def gemm_set_reserved_sms(self, n):
            seen.append(("own", n))

    monkeypatch.setattr(K, "_cuda", lambda: FakeExt())
    monkeypatch.setattr(torch._C, "_set_sm_carveout_experimental", lambda n: seen.append(("lib", n)), raising=False)
    monkeypatch.setattr(K, "LIB_CARVEOUT", True)
    K.set_reserved_sms(16)
    K.set_reserved_sms(0)
    assert seen == [("own", 16), ("lib", 16), ("own", 0), ("lib", None)]
    seen.clear()
    monkeypatch.setattr(K, "LIB_CARVEOUT", False)
    K.set_reserved_sms(16)
    assert seen == [("own", 16)]


def test_library_route_rejects_what_it_cannot_do():
    """impl="library" takes plain GEMMs only, and impl must name a route."""
    a = mx_quantize_ref(torch.randn(64, 64).to(torch.bfloat16))
    b = mx_quantize_ref(torch.randn(32, 64).to(torch.bfloat16))
    with pytest.raises(ValueError):
        gemm_mxfp8(a, b, impl="library")  # CPU operands: not eligible
    with pytest.raises(ValueError):
        gemm_mxfp8(a, b, impl="cublas")
