"""The MXFP8 branches of the fused GPT blocks (``AttnBlockFn`` / ``MLPBlockFn`` with
``recipe="mx"``), run on the CPU with stand-ins for the sm_100a kernels: the
block-scaled GEMM becomes the PyTorch oracle of the dequantised operands with the
same epilogue (bias, residual, GELU, dGELU, fp32 accumulate), attention the fp32
reference, LayerNorm backward / column sums plain PyTorch.  The MX quantisers run
their reference path.  Forward outputs and every gradient (input, weights, biases,
LayerNorm affine) are compared with fp32 autograd of the unquantised block: a
transposed operand or a row-wise / column-wise mix-up would miss by far more than
the few percent that E4M3 / E5M2 with 1x32 scales cost."""
import math

import pytest
import torch
import torch.nn.functional as F

import mtorus.ops.attention as A
import mtorus.ops.fused as FU
import mtorus.ops.kernels as K
import mtorus.ops.mxfp8 as MX

B, S, H, DH = 2, 128, 1, 128
D, FF = H * DH, 256
T = B * S


def _gelu_grad(x):
    cdf = 0.5 * (1.0 + torch.erf(x / math.sqrt(2.0)))
    return cdf + x * torch.exp(-0.5 * x * x) / math.sqrt(2.0 * math.pi)


def _gemm_mx_oracle(a, b, out=None, *, bias=None, residual=None, act=None, aux=None, alpha=None, accumulate=False,
                    out_dtype=torch.bfloat16):
    y = MX.gemm_mxfp8_ref(a, b)
    if alpha is not None:
        y = y * float(alpha)
    if bias is not None:
        y = y + bias
    if aux is not None:
        y = y * _gelu_grad(aux.float())
    if out is None:
        out = torch.empty(y.shape, dtype=out_dtype)
    if out.dtype == torch.float32:
        if accumulate:
            out += y
        else:
            out.copy_(y)
        return out
    if residual is not None:
        y = y + residual.float()
    out.copy_(y.to(torch.bfloat16))
    if act is not None:
        act.copy_(F.gelu(out.float()).to(torch.bfloat16))
    return out


def _attn_fwd(qkv, b, s, h, drop=None):
    return A.reference_attention(qkv, b, s, h, DH).to(torch.bfloat16), torch.zeros(b, h, s)


def _attn_bwd(do, qkv, o, lse, b, s, h, drop=None, dq_out=None):
    with torch.enable_grad():  # called from inside a custom Function's backward
        q = qkv.float().detach().requires_grad_(True)
        A.reference_attention(q, b, s, h, DH).backward(do.float())
    g = q.grad
    if dq_out is not None:  # the kernel's contract: dQ in fp32 there, the dq third unwritten
        dq_out.copy_(g[:, :dq_out.shape[1]])
        g = g.clone()
        g[:, :dq_out.shape[1]] = float("nan")
    return g.to(torch.bfloat16)


def _colsum(x, out, accumulate, scale=None):
    s = x.float().sum(0)
    if accumulate:
        out += s
    else:
        out.copy_(s)
    return out


def _ln_bwd(dy, x, gamma, mean, rstd, dgamma, dbeta, accumulate, dres=None):
    with torch.enable_grad():
        xf = x.float().detach().requires_grad_(True)
        g = gamma.detach().clone().requires_grad_(True)
        bt = torch.zeros_like(g, requires_grad=True)
        F.layer_norm(xf, (x.shape[-1],), g, bt, 1e-5).backward(dy.float())
    for dst, src in ((dgamma, g.grad), (dbeta, bt.grad)):
        if accumulate:
            dst += src
        else:
            dst.copy_(src)
    dx = xf.grad + (0 if dres is None else dres.float())
    return dx.to(torch.bfloat16)


class _P:
    """A parameter as the fused blocks see it: fp32 data, fp32 main_grad, and the
    MX encodings of its bf16 copy (what refresh_fp8_weights produces)."""

    def __init__(self, t, quantize=False):
        self.data = t
        self.main_grad = torch.zeros_like(t, dtype=torch.float32)
        self.shape = t.shape
        if quantize:
            self.mx = MX.mx_quantize_rc(t.to(torch.bfloat16), MX.E4M3)


@pytest.fixture
def cpu_kernels(monkeypatch):
    monkeypatch.setattr(MX, "gemm_mxfp8", _gemm_mx_oracle)
    monkeypatch.setattr(A, "attention_fwd", _attn_fwd)
    monkeypatch.setattr(A, "attention_bwd", _attn_bwd)
    monkeypatch.setattr(K, "colsum_", _colsum)
    monkeypatch.setattr(K, "layernorm_bwd", _ln_bwd)
    FU.FusedGradState.accumulate = False
    FU.FusedGradState.grad_ready_hook = None
    st = type("St", (), {"recipe": "mx"})()
    yield (st, "L0")


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


def _ln_params():
    g = torch.Generator().manual_seed(11)
    return _P(1.0 + 0.1 * torch.randn(D, generator=g)), _P(0.1 * torch.randn(D, generator=g))


def test_attention_block_mx_branch_matches_fp32_autograd(cpu_kernels):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(T, D, generator=g).to(torch.bfloat16)
    wq, bq = _P(0.05 * torch.randn(3 * D, D, generator=g), True), _P(0.01 * torch.randn(3 * D, generator=g))
    wo, bo = _P(0.05 * torch.randn(D, D, generator=g), True), _P(0.01 * torch.randn(D, generator=g))
    gamma, beta = _ln_params()
    xin = x.clone().requires_grad_(True)
    out = FU.AttnBlockFn.apply(xin, (gamma, beta, 1e-5), (wq, bq), (wo, bo), (B, S, H, DH), cpu_kernels)
    dout = (0.1 * torch.randn(T, D, generator=g)).to(torch.bfloat16)
    out.backward(dout)

    # fp32 reference of the same block
    xr = x.float().requires_grad_(True)
    P = {k: v.data.clone().requires_grad_(True) for k, v in
         dict(wq=wq, bq=bq, wo=wo, bo=bo, gamma=gamma, beta=beta).items()}
    h = F.layer_norm(xr, (D,), P["gamma"], P["beta"], 1e-5)
    o = A.reference_attention(h @ P["wq"].t() + P["bq"], B, S, H, DH)
    ref = o @ P["wo"].t() + P["bo"] + xr
    ref.backward(dout.float())

    assert _rel(out.detach(), ref.detach()) < 0.03
    assert _rel(xin.grad, xr.grad) < 0.1
    for name, p in dict(wq=wq, bq=bq, wo=wo, bo=bo, gamma=gamma, beta=beta).items():
        assert _rel(p.main_grad, P[name].grad) < 0.1, name


def test_mlp_block_mx_branch_matches_fp32_autograd(cpu_kernels):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(T, D, generator=g).to(torch.bfloat16)
    w1, b1 = _P(0.05 * torch.randn(FF, D, generator=g), True), _P(0.01 * torch.randn(FF, generator=g))
    w2, b2 = _P(0.05 * torch.randn(D, FF, generator=g), True), _P(0.01 * torch.randn(D, generator=g))
    gamma, beta = _ln_params()
    xin = x.clone().requires_grad_(True)
    out = FU.MLPBlockFn.apply(xin, (gamma, beta, 1e-5), (w1, b1, w2, b2), cpu_kernels)
    dout = (0.1 * torch.randn(T, D, generator=g)).to(torch.bfloat16)
    out.backward(dout)

    xr = x.float().requires_grad_(True)
    P = {k: v.data.clone().requires_grad_(True) for k, v in
         dict(w1=w1, b1=b1, w2=w2, b2=b2, gamma=gamma, beta=beta).items()}
    h = F.layer_norm(xr, (D,), P["gamma"], P["beta"], 1e-5)
    ref = F.gelu(h @ P["w1"].t() + P["b1"]) @ P["w2"].t() + P["b2"] + xr
    ref.backward(dout.float())

    assert _rel(out.detach(), ref.detach()) < 0.03
    assert _rel(xin.grad, xr.grad) < 0.1
    for name, p in dict(w1=w1, b1=b1, w2=w2, b2=b2, gamma=gamma, beta=beta).items():
        assert _rel(p.main_grad, P[name].grad) < 0.1, name


def test_model_refreshes_mx_weights_both_ways():
    """GptModel.enable_fp8(recipe="mx") + refresh_fp8_weights(): every block weight gets
    its row-wise (forward) and column-wise (dgrad) encodings of the current bf16 copy."""
    from mtorus.models.gpt import GptConfig, GptModel

    m = GptModel(GptConfig(256, 128, 2, 1, 256, 128, 0.0), init="reference")
    m.flatten(torch.device("cpu"))
    assert m.enable_fp8(16, recipe="mx").recipe == "mx"
    m.refresh_fp8_weights()
    for name, w in m.fp8_weights():
        r, c = w.mx
        assert r.codes.shape == w.shape and c.codes.shape == w.shape[::-1], name
        assert torch.equal(r.codes, MX.mx_quantize_ref(w.w16, MX.E4M3).codes)
        assert torch.equal(c.codes, MX.mx_quantize_ref(w.w16.t().contiguous(), MX.E4M3).codes)
        assert not hasattr(w, "w8")  # the per-tensor copies are not allocated under MX
    with pytest.raises(ValueError):
        m.enable_fp8(16, recipe="block")
