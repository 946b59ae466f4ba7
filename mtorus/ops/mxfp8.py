"""MXFP8: FP8 with one power-of-two scale per 32-element block (OCP microscaling),
for the tcgen05 ``kind::mxf8f6f4`` block-scaled GEMM.

The reference's block quantiser (``to_fp8_per_block``, crates/mt-core/src/precision/
quantize.rs:68-97) keeps one fp32 scale per block of any size on the host.  The
hardware form kept here has 32-element blocks along the GEMM's K dimension and an
8-bit biased exponent (UE8M0) per block, which the tensor core applies inside the
MMA, so a GEMM over block-scaled operands needs no dequantise pass and no epilogue
scale.

Block rule: X = the smallest integer with ``amax <= fmax * 2**X`` (so no element
saturates); the codes are ``fp8(x * 2**-X)`` rounded to nearest even, and the scale
byte is ``X + 127`` (clamped to [0, 254]).  An all-zero block gets X = 0; a block
holding a NaN or an Inf gets the UE8M0 NaN byte 255, which turns every output it
touches into NaN (the overflow check downstream sees it).  ``fmax`` is the
format's largest finite value, 448 (E4M3) or 57344 (E5M2).

Scale layout (what ``tcgen05.cp`` copies into tensor memory): for an operand of
R rows and K columns the scales form atoms of 128 rows x 4 K-blocks (512 bytes),
stored row-block-major ``[ceil(R/128)][ceil(K/128)][512]``; inside an atom the
scale of row r and K-block j sits at byte ``(r % 32) * 16 + (r % 128 // 32) * 4 + j % 4``.
Padding rows and K-blocks hold 127 (a scale of 1).

``mx_quantize_ref`` / ``mx_dequantize`` are plain PyTorch on any device (the oracle
for the CUDA quantiser and GEMM); ``mx_quantize`` and ``gemm_mxfp8`` run the sm_100a
kernels on CUDA tensors.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .._ext import cuda as _cuda

E4M3, E5M2 = 0, 1
MX_FMT_MAX = {E4M3: 448.0, E5M2: 57344.0}
_TORCH_FP8 = {E4M3: torch.float8_e4m3fn, E5M2: torch.float8_e5m2}
BLOCK = 32


def sf_numel(rows: int, k: int) -> int:
    """Bytes of the scale tensor of a [rows, k] operand."""
    return (rows + 127) // 128 * ((k + 127) // 128) * 512


def sf_offsets(rows: int, k: int, device=None) -> torch.Tensor:
    """int64 [rows, k // 32]: byte offset of each block's scale in the atom layout."""
    nkb4 = (k + 127) // 128
    r = torch.arange(rows, device=device, dtype=torch.int64)[:, None]
    j = torch.arange(k // BLOCK, device=device, dtype=torch.int64)[None, :]
    return ((r // 128) * nkb4 + j // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + j % 4


@dataclass
class MxTensor:
    """Block-scaled FP8 operand: ``codes`` uint8 [R, K], ``sf`` uint8 atoms, format id."""
    codes: torch.Tensor
    sf: torch.Tensor
    fmt: int

    @property
    def shape(self):
        return tuple(self.codes.shape)

    def dequantize(self) -> torch.Tensor:
        return mx_dequantize(self)


def _block_exponent(amax: torch.Tensor, fmax: float) -> torch.Tensor:
    """Smallest integer X with amax <= fmax * 2**X, from the IEEE-754 fields (exact)."""
    fbits = torch.tensor([fmax], dtype=torch.float32).view(torch.int32).item()
    ef, mf = (fbits >> 23) & 0xFF, fbits & 0x7FFFFF
    ua = amax.contiguous().view(torch.int32)
    ea, ma = (ua >> 23) & 0xFF, ua & 0x7FFFFF
    x = ea - ef + (ma > mf).to(torch.int32)
    x = x.clamp(-127, 127)
    return torch.where(amax > 0, x, torch.zeros_like(x))


def mx_quantize_ref(x: torch.Tensor, fmt: int = E4M3, fmax: Optional[float] = None) -> MxTensor:
    """Plain-PyTorch MXFP8 quantisation of a 2-D tensor (K a multiple of 32)."""
    if x.dim() != 2 or x.shape[1] % BLOCK:
        raise ValueError("mx_quantize: 2-D input with K a multiple of 32 expected")
    fmax = float(MX_FMT_MAX[fmt] if fmax is None else fmax)
    R, K = x.shape
    xb = x.float().reshape(R, K // BLOCK, BLOCK)
    amax = xb.abs().amax(-1)
    finite = torch.isfinite(xb).all(-1)
    amax = torch.where(finite, amax, torch.zeros_like(amax))
    X = _block_exponent(amax, fmax)
    inv = torch.ldexp(torch.ones_like(amax), (-X).float())
    scaled = (xb * inv[..., None]).reshape(R, K)
    codes = scaled.to(_TORCH_FP8[fmt]).view(torch.uint8)
    sf = torch.full((sf_numel(R, K),), 127, dtype=torch.uint8, device=x.device)
    byte = torch.where(finite, X + 127, torch.full_like(X, 255)).to(torch.uint8)
    sf[sf_offsets(R, K, x.device).reshape(-1)] = byte.reshape(-1)
    return MxTensor(codes.contiguous(), sf, int(fmt))


def mx_dequantize(t: MxTensor) -> torch.Tensor:
    """fp32 values of a block-scaled operand (NaN where the scale byte is 255)."""
    R, K = t.codes.shape
    vals = t.codes.view(_TORCH_FP8[t.fmt]).float().reshape(R, K // BLOCK, BLOCK)
    byte = t.sf[sf_offsets(R, K, t.codes.device)].to(torch.int32)
    scale = torch.ldexp(torch.ones(byte.shape, device=byte.device), (byte - 127).float())
    scale = torch.where(byte == 255, torch.full_like(scale, float("nan")), scale)
    return (vals * scale[..., None]).reshape(R, K)


def mx_quantize(x: torch.Tensor, fmt: int = E4M3, fmax: Optional[float] = None) -> MxTensor:
    """MXFP8 quantisation: the sm_100a kernel for CUDA tensors, the reference on the CPU."""
    if not x.is_cuda:
        return mx_quantize_ref(x, fmt, fmax)
    if x.dim() != 2 or x.shape[1] % BLOCK:
        raise ValueError("mx_quantize: 2-D input with K a multiple of 32 expected")
    fmax = float(MX_FMT_MAX[fmt] if fmax is None else fmax)
    x = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
    if x.stride(1) != 1:
        x = x.contiguous()
    R, K = x.shape
    codes = torch.empty((R, K), dtype=torch.uint8, device=x.device)
    sf = torch.empty(sf_numel(R, K), dtype=torch.uint8, device=x.device)
    _cuda().mx_quantize(x, codes, sf, int(fmt), fmax)
    return MxTensor(codes, sf, int(fmt))


def _library_default() -> bool:
    import os

    return os.environ.get("MTORUS_MX_LIBRARY_GEMM", "1") != "0"


# Plain block-scaled GEMMs (no epilogue beyond a bias, a fresh bf16 / fp32 output) go to
# cuBLASLt's MXFP8 kernel through torch._scaled_mm when this is set (the default;
# MTORUS_MX_LIBRARY_GEMM=0 keeps every GEMM on gemm_2sm_kernel).  Measured on B200 at the
# GPT-1B shapes, with results bit-identical to the CTA-pair kernel: QKV forward 0.247 ->
# 0.147 ms, FFN1 dgrad 0.268 -> 0.181, FFN1 wgrad 0.300 -> 0.207.  cuBLASLt reaches a
# higher tensor-pipe duty on these plain tiles; the fused epilogues (residual add, GELU /
# dGELU, MX-output codes, fp32 accumulation, dropout) stay on this library's kernel.
LIBRARY_PLAIN_GEMM = _library_default()


def _library_residual_default() -> bool:
    import os

    return os.environ.get("MTORUS_MX_LIBRARY_RESIDUAL", "1") != "0"


# A GEMM with a residual add and a long contraction (K >= LIBRARY_RESIDUAL_MIN_K: the FFN2
# forward, 16384 x 2048 x 8192) also runs in the library, followed by a bf16 add of the
# residual: the library GEMM saves more than the add's extra pass over three [M, N] bf16
# tensors costs.  At K = 2048 (the attention output projection) it does not, and the own
# kernel's fused epilogue stays.  The split rounds the GEMM result to bf16 before the add.
LIBRARY_RESIDUAL = _library_residual_default()
LIBRARY_RESIDUAL_MIN_K = 4096


def _library_eligible(a, b, out, residual, act, aux, alpha, accumulate) -> bool:
    from .kernels import gemm_dropout

    return (residual is None and act is None and aux is None and alpha is None and not accumulate
            and not gemm_dropout.armed and out.dtype in (torch.bfloat16, torch.float32)
            and out.is_contiguous() and a.codes.is_cuda and b.codes.shape[0] % 16 == 0
            and all(t.data_ptr() % 16 == 0 for t in (a.codes, b.codes, out)))


def gemm_mxfp8(a: MxTensor, b: MxTensor, out: Optional[torch.Tensor] = None, *, bias=None, residual=None,
               act=None, aux=None, alpha=None, accumulate: bool = False,
               out_dtype: torch.dtype = torch.bfloat16, impl: str = "auto") -> torch.Tensor:
    """out[M, N] = epilogue(alpha * A . B^T) with A [M, K] and B [N, K] block-scaled
    (both K-major); epilogue as in ``ops.kernels.gemm`` (bias, residual, GELU / dGELU,
    fp32 accumulate).  ``impl``: "own" runs gemm_2sm_kernel, "library" cuBLASLt's MXFP8
    GEMM (plain GEMMs only; the bias is rounded to the output dtype, as cuBLASLt adds it
    in that precision), "auto" the library for plain GEMMs when ``LIBRARY_PLAIN_GEMM`` and
    for residual GEMMs with K >= ``LIBRARY_RESIDUAL_MIN_K`` when ``LIBRARY_RESIDUAL`` too."""
    M, K = a.codes.shape
    N, Kb = b.codes.shape
    if K != Kb:
        raise ValueError(f"gemm_mxfp8: K mismatch {K} vs {Kb}")
    if impl not in ("auto", "own", "library"):
        raise ValueError(f"gemm_mxfp8: impl must be auto, own or library, not {impl!r}")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.codes.device)
    eligible = _library_eligible(a, b, out, residual, act, aux, alpha, accumulate)
    if (impl == "auto" and LIBRARY_PLAIN_GEMM and LIBRARY_RESIDUAL and residual is not None
            and K >= LIBRARY_RESIDUAL_MIN_K and out.dtype == torch.bfloat16 and residual.dtype == torch.bfloat16
            and residual.shape == out.shape
            and _library_eligible(a, b, out, None, act, aux, alpha, accumulate)):
        y = gemm_mxfp8(a, b, torch.empty_like(out), bias=bias, impl="library")
        return torch.add(y, residual, out=out)
    if impl == "library" and not eligible:
        raise ValueError("gemm_mxfp8: the library path takes plain GEMMs only (bias at most, no accumulate)")
    if impl == "library" or (impl == "auto" and eligible and LIBRARY_PLAIN_GEMM):
        sa = a.sf.view(torch.float8_e8m0fnu).reshape((M + 127) // 128 * 128, -1)
        sb = b.sf.view(torch.float8_e8m0fnu).reshape((N + 127) // 128 * 128, -1)
        torch._scaled_mm(a.codes.view(_TORCH_FP8[a.fmt]), b.codes.view(_TORCH_FP8[b.fmt]).t(), sa, sb,
                         bias=None if bias is None else bias.to(out.dtype), out_dtype=out.dtype, out=out)
        return out
    _cuda().gemm_mxfp8(a.codes, a.fmt, a.sf, b.codes, b.fmt, b.sf, out, bias, residual, act, aux, alpha,
                       bool(accumulate))
    return out


def gemm_mxfp8_mx_out(a: MxTensor, b: MxTensor, fmt: int, out: Optional[torch.Tensor] = None, *, bias=None,
                      aux=None, alpha=None, gelu: bool = False, colsum: Optional[torch.Tensor] = None,
                      accumulate: bool = True, store_d: bool = True, fmax: Optional[float] = None):
    """The block-scaled GEMM whose epilogue quantises its own output: D = epilogue(alpha
    * A . B^T) (bias, dGELU with ``aux``), then the bf16-rounded D -- or GELU of it when
    ``gelu`` -- as MXFP8 row codes [M, N] and column codes [N, M], exactly what
    ``mx_quantize_rc`` makes of that bf16 tensor, without writing it.  ``colsum``
    (fp32 [N], optional) receives its column sums (added when ``accumulate``).  D is
    stored in bf16 only when ``store_d`` (the pre-activation a dGELU needs later).
    M and N multiples of 128.  Returns (D or None, rows, cols).  The CPU path is the
    unfused oracle."""
    M, K = a.codes.shape
    N, Kb = b.codes.shape
    if K != Kb:
        raise ValueError(f"gemm_mxfp8_mx_out: K mismatch {K} vs {Kb}")
    if M % 128 or N % 128:
        raise ValueError("gemm_mxfp8_mx_out: M and N must be multiples of 128")
    fmax = float(MX_FMT_MAX[fmt] if fmax is None else fmax)
    dev = a.codes.device
    if not a.codes.is_cuda:
        d = gemm_mxfp8_ref(a, b)
        if alpha is not None:
            d = d * alpha.float()
        if bias is not None:
            d = d + bias.float()
        if aux is not None:  # dGELU: d * GELU'(aux), the erf GELU's derivative
            x = aux.float()
            d = d * (0.5 * (1.0 + torch.erf(x * 0.7071067811865476)) + x * torch.exp(-0.5 * x * x) * 0.3989422804014327)
        d16 = d.to(torch.bfloat16)
        src = d16
        if gelu:
            src = torch.nn.functional.gelu(d16.float()).to(torch.bfloat16)
        if colsum is not None:
            cs = src.float().sum(0)
            if accumulate:
                colsum += cs
            else:
                colsum.copy_(cs)
        if out is not None and store_d:
            out.copy_(d16)
        return (out if store_d else None), mx_quantize_ref(src, fmt, fmax), mx_quantize_ref(src.t(), fmt, fmax)
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    rc = torch.empty((M, N), dtype=torch.uint8, device=dev)
    cc = torch.empty((N, M), dtype=torch.uint8, device=dev)
    rsf = torch.empty(sf_numel(M, N), dtype=torch.uint8, device=dev)
    csf = torch.empty(sf_numel(N, M), dtype=torch.uint8, device=dev)
    if colsum is not None and not accumulate:
        colsum.zero_()
    _cuda().gemm_mxfp8(a.codes, a.fmt, a.sf, b.codes, b.fmt, b.sf, out, bias, None, None, aux, alpha, False,
                       out_rc=rc, out_rsf=rsf, out_cc=cc, out_csf=csf, out_fmt=int(fmt), out_fmax=fmax,
                       out_colsum=colsum, out_gelu=bool(gelu), store_d=bool(store_d))
    return (out if store_d else None), MxTensor(rc, rsf, int(fmt)), MxTensor(cc, csf, int(fmt))


_RC_ACT = {None: 0, "gelu": 2, "dgelu": 3}


def _erf_gelu(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * x * (1.0 + torch.erf(x * 0.7071067811865476))


def _erf_gelu_grad(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * (1.0 + torch.erf(x * 0.7071067811865476)) + x * torch.exp(-0.5 * x * x) * 0.3989422804014327


def mx_quantize_rc(x: torch.Tensor, fmt: int = E4M3, fmax: Optional[float] = None,
                   colsum: Optional[torch.Tensor] = None, accumulate: bool = True,
                   xq: Optional[torch.Tensor] = None, act: Optional[str] = None,
                   aux: Optional[torch.Tensor] = None):
    """Row-wise MXFP8 of x [R, C] (32-blocks along C) and of its transpose [C, R]
    (32-blocks along R), in one pass on the GPU: the operands that contract over C
    and over R.  R and C multiples of 32.  The reference on the CPU.

    colsum (fp32 [C], optional): receives the column sums of what is quantised in the
    same pass (the bias gradient when x is a layer's output gradient), added to its
    contents when ``accumulate``, else overwriting them.  xq (fp32 [R, Q], Q a multiple of
    128, optional): the first Q columns are taken from xq rounded to bf16 instead of from x.
    act: None quantises x; "gelu" bf16(GELU(x)) (x a pre-activation); "dgelu"
    bf16(x * GELU'(aux)) with aux the bf16 pre-activation [R, C] (x the gradient of the
    GELU output)."""
    if x.dim() != 2 or x.shape[0] % BLOCK or x.shape[1] % BLOCK:
        raise ValueError("mx_quantize_rc: 2-D input with both sizes multiples of 32 expected")
    if act not in _RC_ACT:
        raise ValueError(f"mx_quantize_rc: act must be None, 'gelu' or 'dgelu', not {act!r}")
    if (act == "dgelu") != (aux is not None):
        raise ValueError("mx_quantize_rc: aux is the pre-activation of act='dgelu' and nothing else")
    if act is not None and xq is not None:
        raise ValueError("mx_quantize_rc: xq takes no activation")
    if act is not None and not x.is_cuda:
        xf = x.to(torch.bfloat16).float()
        xf = _erf_gelu(xf) if act == "gelu" else xf * _erf_gelu_grad(aux.to(torch.bfloat16).float())
        x, act, aux = xf.to(torch.bfloat16), None, None
    if xq is not None:
        if xq.shape[0] != x.shape[0] or xq.shape[1] % 128 or xq.shape[1] > x.shape[1]:
            raise ValueError("mx_quantize_rc: xq must be [R, Q] with Q a multiple of 128, Q <= C")
        if not x.is_cuda:
            x = x.clone()
            x[:, :xq.shape[1]] = xq.to(x.dtype)
            xq = None
    if not x.is_cuda:
        if colsum is not None:
            cs = x.float().sum(0)
            if accumulate:
                colsum += cs
            else:
                colsum.copy_(cs)
        return mx_quantize_ref(x, fmt, fmax), mx_quantize_ref(x.t(), fmt, fmax)
    fmax = float(MX_FMT_MAX[fmt] if fmax is None else fmax)
    x = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
    if x.stride(1) != 1:
        x = x.contiguous()
    R, C = x.shape
    rc = torch.empty((R, C), dtype=torch.uint8, device=x.device)
    cc = torch.empty((C, R), dtype=torch.uint8, device=x.device)
    rsf = torch.empty(sf_numel(R, C), dtype=torch.uint8, device=x.device)
    csf = torch.empty(sf_numel(C, R), dtype=torch.uint8, device=x.device)
    if colsum is not None and not accumulate:
        colsum.zero_()
    if aux is not None:
        aux = aux if aux.dtype == torch.bfloat16 else aux.to(torch.bfloat16)
        if aux.stride(1) != 1:
            aux = aux.contiguous()
    _cuda().mx_quantize_rc(x, rc, rsf, cc, csf, int(fmt), fmax, colsum, xq, _RC_ACT[act], aux)
    return MxTensor(rc, rsf, int(fmt)), MxTensor(cc, csf, int(fmt))


def mx_layernorm_rc(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5,
                    fmt: int = E4M3, fmax: Optional[float] = None):
    """LayerNorm of x [R, d] straight into MXFP8, row-wise ([R, d]) and column-wise
    ([d, R]), plus the fp32 mean / rstd rows for the backward; no bf16 output (CUDA,
    R and d multiples of 32: a row-statistics kernel, then the tile quantiser with
    the normalisation applied on load).  Elsewhere: LayerNorm, rounded to bf16, then
    ``mx_quantize_rc``."""
    R, d = x.shape
    if x.is_cuda and x.dtype == torch.bfloat16 and R % 32 == 0 and d % 32 == 0:
        fmax = float(MX_FMT_MAX[fmt] if fmax is None else fmax)
        x = x.contiguous()
        dev = x.device
        rc = torch.empty((R, d), dtype=torch.uint8, device=dev)
        cc = torch.empty((d, R), dtype=torch.uint8, device=dev)
        rsf = torch.empty(sf_numel(R, d), dtype=torch.uint8, device=dev)
        csf = torch.empty(sf_numel(d, R), dtype=torch.uint8, device=dev)
        mean = torch.empty(R, dtype=torch.float32, device=dev)
        rstd = torch.empty(R, dtype=torch.float32, device=dev)
        _cuda().layernorm_fwd_mx_rc(x, gamma.float().contiguous(), beta.float().contiguous(), float(eps), rc, rsf,
                                    cc, csf, mean, rstd, int(fmt), fmax)
        return MxTensor(rc, rsf, int(fmt)), MxTensor(cc, csf, int(fmt)), mean, rstd
    xf = x.float()
    mean = xf.mean(-1)
    rstd = torch.rsqrt(xf.var(-1, unbiased=False) + eps)
    h = ((xf - mean[:, None]) * rstd[:, None] * gamma.float() + beta.float()).to(torch.bfloat16)
    r, c = mx_quantize_rc(h, fmt, fmax)
    return r, c, mean, rstd


def _mm(a: MxTensor, b: MxTensor, out_dtype, bias=None) -> torch.Tensor:
    if a.codes.is_cuda:
        return gemm_mxfp8(a, b, bias=bias, out_dtype=out_dtype)
    y = gemm_mxfp8_ref(a, b)
    return (y if bias is None else y + bias).to(out_dtype)


class MxLinearFn(torch.autograd.Function):
    """y = x . W^T + b with all three GEMMs block-scaled (the MXFP8 training recipe):
    E4M3 activations and weights, E5M2 output gradients, 1x32 UE8M0 scales along each
    GEMM's contraction dimension, fp32 accumulation.  Forward: row-wise x and W.
    dgrad: row-wise dY with column-wise W.  wgrad: column-wise dY with column-wise x.
    Each tensor is quantised once, both ways, by ``mx_quantize_rc``.  CUDA tensors run
    the sm_100a kernels; CPU tensors run the PyTorch oracle with the same numerics.
    x [T, in], W [out, in] (T, in, out multiples of 32), b fp32 [out] or None."""

    @staticmethod
    def forward(ctx, x, w, b):
        x2 = x.reshape(-1, x.shape[-1])
        xr, xc = mx_quantize_rc(x2.to(torch.bfloat16), E4M3)
        wr, wc = mx_quantize_rc(w.to(torch.bfloat16), E4M3)
        y = _mm(xr, wr, torch.bfloat16, None if b is None else b.float())
        ctx.save_for_backward(xc.codes, xc.sf, wc.codes, wc.sf)
        ctx.has_bias = b is not None
        ctx.x_shape, ctx.w_dtype = x.shape, w.dtype
        return y.reshape(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        xc_codes, xc_sf, wc_codes, wc_sf = ctx.saved_tensors
        xc, wc = MxTensor(xc_codes, xc_sf, E4M3), MxTensor(wc_codes, wc_sf, E4M3)
        dy2 = dy.reshape(-1, dy.shape[-1]).to(torch.bfloat16)
        dyr, dyc = mx_quantize_rc(dy2, E5M2)
        dx = _mm(dyr, wc, torch.bfloat16).reshape(ctx.x_shape)
        dw = _mm(dyc, xc, torch.float32).to(ctx.w_dtype)
        db = dy2.float().sum(0) if ctx.has_bias else None
        return dx, dw, db


def mx_linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Block-scaled FP8 linear layer (see MxLinearFn)."""
    return MxLinearFn.apply(x, w, b)


def enable_mx_linears(module: torch.nn.Module) -> int:
    """Run every Linear of ``module`` through ``mx_linear`` (the MXFP8 recipe: all three
    GEMMs block-scaled).  A call whose token count, input or output width is not a
    multiple of 32 runs the layer's own forward instead.  Works on any device (CUDA
    kernels on the GPU, the oracle on the CPU).  Returns the number of layers converted."""
    import torch.nn.functional as F

    n = 0
    for mod in module.modules():
        w = getattr(mod, "weight", None)
        if not isinstance(w, torch.nn.Parameter) or w.dim() != 2 or not hasattr(mod, "bias"):
            continue
        if isinstance(mod, torch.nn.Embedding) or type(mod).__name__ == "Embedding":
            continue

        def fwd(x, mod=mod):
            T = x.numel() // x.shape[-1]
            out_f, in_f = mod.weight.shape
            b = None if mod.bias is None else mod.bias
            if T % BLOCK or in_f % BLOCK or out_f % BLOCK:
                return F.linear(x, mod.weight.to(x.dtype), None if b is None else b.to(x.dtype))
            return mx_linear(x, mod.weight, b).to(x.dtype)

        mod.forward = fwd
        n += 1
    return n


def gemm_mxfp8_ref(a: MxTensor, b: MxTensor) -> torch.Tensor:
    """fp32 oracle of ``gemm_mxfp8``: the product of the dequantised operands."""
    return mx_dequantize(a) @ mx_dequantize(b).t()


__all__ = ["E4M3", "E5M2", "MX_FMT_MAX", "MxTensor", "sf_numel", "sf_offsets", "mx_quantize", "mx_quantize_ref",
           "mx_quantize_rc", "mx_layernorm_rc", "mx_dequantize", "gemm_mxfp8", "gemm_mxfp8_mx_out", "gemm_mxfp8_ref", "MxLinearFn", "mx_linear", "enable_mx_linears"]
