"""Autograd functions that route the GPT hot path through the sm_100a kernels.

The functions take the *parameters* as non-differentiable arguments (wrapped in
a tuple) and write parameter gradients straight into each parameter's fp32
``main_grad`` view of the flat gradient buffer (see ``mtorus.parallel.flat``):
the wgrad GEMM epilogue stores / accumulates fp32, so there is no bf16 grad
tensor, no AccumulateGrad kernel and no extra pass before the optimizer.

``FusedGradState.accumulate`` is False on the first micro-batch of a step (the
kernels overwrite ``main_grad``) and True afterwards (they add into it).
"""
from __future__ import annotations

from typing import Optional

import torch
from torch.autograd import Function

from . import fp8 as F8
from . import kernels as K


class FusedGradState:
    accumulate: bool = False
    # called as hook(param_list) after the gradients of those params are final for
    # this backward pass (used by the data-parallel bucket scheduler)
    grad_ready_hook = None


def _grads_done(*params):
    hook = FusedGradState.grad_ready_hook
    if hook is not None:
        hook([p for p in params if p is not None])


class LayerNormFn(Function):
    """y = LayerNorm(x) with fp32 gamma/beta; reference: Burn LayerNorm (eps 1e-5)."""

    @staticmethod
    def forward(ctx, x, params, eps):
        gamma, beta = params
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        y, mean, rstd = K.layernorm_fwd(x2, gamma.data, beta.data, eps)
        ctx.save_for_backward(x2, mean, rstd)
        ctx.params = params
        return y.view(shp)

    @staticmethod
    def backward(ctx, dy):
        x2, mean, rstd = ctx.saved_tensors
        gamma, beta = ctx.params
        dx = K.layernorm_bwd(dy.reshape(x2.shape), x2, gamma.data, mean, rstd, gamma.main_grad,
                             beta.main_grad, FusedGradState.accumulate)
        _grads_done(gamma, beta)
        return dx.view(dy.shape), None, None


class LinearFn(Function):
    """y = x W^T + b (+ residual); reference: Burn Linear (transformer.rs:34-37,84)."""

    @staticmethod
    def forward(ctx, x, residual, params):
        w, b = params
        y = K.gemm(x, w.w16, bias=None if b is None else b.data, residual=residual)
        ctx.save_for_backward(x)
        ctx.params = params
        ctx.has_res = residual is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        w, b = ctx.params
        dy = dy.contiguous()
        acc = FusedGradState.accumulate
        dx = K.gemm(dy, w.w16, b_mn=True)
        K.gemm(dy, x, out=w.main_grad, a_mn=True, b_mn=True, accumulate=acc)
        if b is not None:
            K.colsum_(dy, b.main_grad, acc)
        _grads_done(w, b)
        return dx, (dy if ctx.has_res else None), None


class MLPFn(Function):
    """out = residual + W2 GELU(W1 h + b1) + b2 with GELU and dGELU fused into the
    GEMM epilogues (reference FeedForward, transformer.rs:89-110)."""

    @staticmethod
    def forward(ctx, h, residual, params):
        w1, b1, w2, b2 = params
        T = h.shape[0]
        F = w1.shape[0]
        pre = torch.empty((T, F), dtype=torch.bfloat16, device=h.device)
        act = torch.empty_like(pre)
        K.gemm(h, w1.w16, out=pre, bias=b1.data, act=act)
        out = K.gemm(act, w2.w16, bias=b2.data, residual=residual)
        ctx.save_for_backward(h, pre, act)
        ctx.params = params
        return out

    @staticmethod
    def backward(ctx, dout):
        h, pre, act = ctx.saved_tensors
        w1, b1, w2, b2 = ctx.params
        dout = dout.contiguous()
        acc = FusedGradState.accumulate
        # dpre = (dout W2) * gelu'(pre)
        dpre = K.gemm(dout, w2.w16, b_mn=True, aux=pre)
        K.gemm(dout, act, out=w2.main_grad, a_mn=True, b_mn=True, accumulate=acc)
        K.colsum_(dout, b2.main_grad, acc)
        _grads_done(w2, b2)
        dh = K.gemm(dpre, w1.w16, b_mn=True)
        K.gemm(dpre, h, out=w1.main_grad, a_mn=True, b_mn=True, accumulate=acc)
        K.colsum_(dpre, b1.main_grad, acc)
        _grads_done(w1, b1)
        return dh, dout, None


_ANCHOR = {}


def grad_anchor(device) -> torch.Tensor:
    """An empty leaf that requires grad: makes the embedding output part of the
    autograd graph although its only tensor input (token ids) is integer."""
    key = str(device)
    if key not in _ANCHOR:
        _ANCHOR[key] = torch.empty(0, device=device, requires_grad=True)
    return _ANCHOR[key]


def _ln_fwd(x2d, ln):
    gamma, beta, eps = ln
    return K.layernorm_fwd(x2d, gamma.data, beta.data, eps)


def _ln_bwd(dh, x2d, mean, rstd, ln, dres):
    gamma, beta, _ = ln
    dx = K.layernorm_bwd(dh, x2d, gamma.data, mean, rstd, gamma.main_grad, beta.main_grad,
                         FusedGradState.accumulate, dres=dres)
    _grads_done(gamma, beta)
    return dx


def _mx(fp8) -> bool:
    """True when the block GEMMs run the MXFP8 recipe (GptModel.enable_fp8(recipe="mx"))."""
    return fp8 is not None and getattr(fp8[0], "recipe", "tensor") == "mx"


def _mx_t(codes, sf, fmt):
    from .mxfp8 import MxTensor

    return MxTensor(codes, sf, fmt)


class AttnBlockFn(Function):
    """x + out_proj(attention(qkv(LN1(x)))) as one autograd node (reference
    TransformerBlock first half, transformer.rs:144-149).  LayerNorm, the QKV and
    output GEMMs (bias + residual in the epilogue) are sm_100a kernels; the LN
    backward adds the residual gradient in the same kernel."""

    @staticmethod
    def forward(ctx, x2d, ln, qkv_params, out_params, shape, fp8=None, drop=None):
        """drop: optional (attention-probability dropout args, attention-output dropout
        args), each (rng, site, thr16, scale)."""
        from .attention import attention_fwd, check_shape

        B, S, H, dh = shape
        check_shape(S, dh)
        wq, bq = qkv_params
        wo, bo = out_params
        ctx.shape = (B, S, H)
        ctx.params = (ln, qkv_params, out_params)
        ctx.fp8 = fp8
        d_probs, d_out = drop if drop is not None else (None, None)
        ctx.drop = (d_probs, d_out)
        if _mx(fp8):
            # MXFP8: every GEMM operand carries 1x32 UE8M0 scales along its contraction dim;
            # inputs are quantised both ways once (row-wise now, column-wise for wgrad)
            from . import mxfp8 as MX

            gamma, beta, eps = ln
            hr, hc, mean, rstd = MX.mx_layernorm_rc(x2d, gamma.data, beta.data, eps, MX.E4M3)
            qkv = MX.gemm_mxfp8(hr, wq.mx[0], bias=bq.data)
            # the attention epilogue writes the output's MX codes both ways beside the bf16 copy
            o, lse, orow, ocol = _attn_fwd_mx(attention_fwd, MX, qkv, B, S, H, d_probs)
            with K.gemm_dropout(d_out, 1):
                out = MX.gemm_mxfp8(orow, wo.mx[0], bias=bo.data, residual=x2d)
            ctx.save_for_backward(x2d, mean, rstd, hc.codes, hc.sf, ocol.codes, ocol.sf, qkv, o, lse)
            return out
        if fp8 is not None:
            st, tag = fp8
            gamma, beta, eps = ln
            # LayerNorm writes the E4M3 codes of the QKV GEMM's input directly
            h8, ih, mean, rstd = st.layernorm_quantize(x2d, gamma.data, beta.data, eps, tag + ".qkv_in", F8.E4M3)
            qkv = F8.gemm_fp8(h8, F8.E4M3, wq.w8, F8.E4M3, bias=bq.data, alpha=ih, alpha2=wq.w8_inv)
            h = h8
        else:
            h, mean, rstd = _ln_fwd(x2d, ln)
            qkv = K.gemm(h, wq.w16, bias=bq.data)
        o, lse = attention_fwd(qkv, B, S, H, d_probs)
        attn_saved = (qkv, o, lse)
        if fp8 is not None:
            o8, io = st.quantize(o, tag + ".out_in", F8.E4M3)
            with K.gemm_dropout(d_out, 1):
                out = F8.gemm_fp8(o8, F8.E4M3, wo.w8, F8.E4M3, bias=bo.data, residual=x2d, alpha=io,
                                  alpha2=wo.w8_inv)
            o = o8
            ctx.inv = (ih, io)
        else:
            with K.gemm_dropout(d_out, 1):
                out = K.gemm(o, wo.w16, bias=bo.data, residual=x2d)
        ctx.save_for_backward(x2d, mean, rstd, h, o, *attn_saved)
        return out

    @staticmethod
    def backward(ctx, dout):
        from .attention import attention_bwd

        if _mx(ctx.fp8):
            return AttnBlockFn._backward_mx(ctx, dout)
        x2d, mean, rstd, h, o, qkv, o_bf16, lse = ctx.saved_tensors
        ln, (wq, bq), (wo, bo) = ctx.params
        dout = dout.contiguous()
        acc = FusedGradState.accumulate
        fp8 = ctx.fp8
        d_probs, d_out = ctx.drop
        # the attention branch's gradient: dout through the output dropout's mask (the
        # residual path keeps dout itself)
        dbr = K.dropout_apply(dout, d_out) if d_out is not None else dout
        if fp8 is not None:
            st, tag = fp8
            ih, io = ctx.inv
            # E5M2 codes and the output-projection bias gradient in one pass over the branch gradient
            g8, ig = st.quantize_colsum(dbr, tag + ".out_grad", F8.E5M2, bo.main_grad, acc)
            do = F8.gemm_fp8(g8, F8.E5M2, wo.w8, F8.E4M3, b_mn=True, alpha=ig, alpha2=wo.w8_inv)
            F8.gemm_fp8(g8, F8.E5M2, o, F8.E4M3, out=wo.main_grad, a_mn=True, b_mn=True, accumulate=acc,
                        alpha=ig, alpha2=io)
        else:
            do = K.gemm(dbr, wo.w16, b_mn=True)
            K.gemm(dbr, o, out=wo.main_grad, a_mn=True, b_mn=True, accumulate=acc)
            K.colsum_(dbr, bo.main_grad, acc)
        _grads_done(wo, bo)
        dqkv = attention_bwd(do, qkv, o_bf16, lse, *ctx.shape, drop=d_probs)
        if fp8 is not None:
            q8, iq = st.quantize_colsum(dqkv, tag + ".qkv_grad", F8.E5M2, bq.main_grad, acc)
            F8.gemm_fp8(q8, F8.E5M2, h, F8.E4M3, out=wq.main_grad, a_mn=True, b_mn=True, accumulate=acc,
                        alpha=iq, alpha2=ih)
            dh = F8.gemm_fp8(q8, F8.E5M2, wq.w8, F8.E4M3, b_mn=True, alpha=iq, alpha2=wq.w8_inv)
        else:
            K.colsum_(dqkv, bq.main_grad, acc)
            K.gemm(dqkv, h, out=wq.main_grad, a_mn=True, b_mn=True, accumulate=acc)
            dh = K.gemm(dqkv, wq.w16, b_mn=True)
        _grads_done(wq, bq)
        return _ln_bwd(dh, x2d, mean, rstd, ln, dout), None, None, None, None, None, None

    @staticmethod
    def _backward_mx(ctx, dout):
        from . import mxfp8 as MX
        from .attention import attention_bwd

        x2d, mean, rstd, hcc, hcs, occ, ocs, qkv, o_bf16, lse = ctx.saved_tensors
        ln, (wq, bq), (wo, bo) = ctx.params
        dout = dout.contiguous()
        acc = FusedGradState.accumulate
        d_probs, d_out = ctx.drop
        dbr = K.dropout_apply(dout, d_out) if d_out is not None else dout
        hc, oc = _mx_t(hcc, hcs, MX.E4M3), _mx_t(occ, ocs, MX.E4M3)
        grow, gcol = MX.mx_quantize_rc(dbr, MX.E5M2, colsum=bo.main_grad, accumulate=acc)
        do = MX.gemm_mxfp8(grow, wo.mx[1])  # dgrad: dY (row) x W (column-wise)
        MX.gemm_mxfp8(gcol, oc, out=wo.main_grad, accumulate=acc)  # wgrad: dY^T x O, both column-wise
        _grads_done(wo, bo)
        # (reading dQ straight from the attention's fp32 accumulator, attention_bwd(dq_out=) with
        # mx_quantize_rc(xq=), moves fewer bytes but measured slower: the fp32 tiles load without
        # the quantiser's prefetch)
        dqkv = attention_bwd(do, qkv, o_bf16, lse, *ctx.shape, drop=d_probs)
        qrow, qcol = MX.mx_quantize_rc(dqkv, MX.E5M2, colsum=bq.main_grad, accumulate=acc)
        MX.gemm_mxfp8(qcol, hc, out=wq.main_grad, accumulate=acc)
        dh = MX.gemm_mxfp8(qrow, wq.mx[1])
        _grads_done(wq, bq)
        return _ln_bwd(dh, x2d, mean, rstd, ln, dout), None, None, None, None, None, None


def _attn_fwd_mx(attention_fwd, MX, qkv, B, S, H, drop):
    """Attention forward plus its output's MXFP8 row / column codes (E4M3): from the kernel's
    epilogue on the GPU, from the separate quantiser where the kernel is replaced."""
    if qkv.is_cuda:
        return attention_fwd(qkv, B, S, H, drop, mx_fmt=MX.E4M3)
    o, lse = attention_fwd(qkv, B, S, H, drop)
    orow, ocol = MX.mx_quantize_rc(o, MX.E4M3)
    return o, lse, orow, ocol


def _mx_gemm_quant(MX, a, b, fmt, out=None, *, bias=None, aux=None, gelu=False, colsum=None, accumulate=True,
                   store_d=True):
    """Block-scaled GEMM whose output (or its GELU, or its product with GELU'(aux))
    leaves as MXFP8 row and column codes.  Returns (D or None, rows, cols).

    On the GPU with ``LIBRARY_PLAIN_GEMM`` (the default) the plain GEMM (bias at most)
    runs in cuBLASLt and writes D in bf16, then the row / column quantiser applies
    GELU / dGELU to each tile as it quantises it: measured on B200 at the GPT-1B FFN
    shapes this pair beats the MX-output epilogue of gemm_2sm_kernel, whose mainloop
    is the slower one.  The epilogue version runs when dropout is drawn in the GEMM
    epilogue or the library path is off; tiles that are not multiples of 128 take this
    library's GEMM with the GELU / dGELU epilogue, then the quantiser."""
    from .kernels import gemm_dropout

    M, N = a.codes.shape[0], b.codes.shape[0]
    if a.codes.is_cuda and MX.LIBRARY_PLAIN_GEMM and not gemm_dropout.armed and M % 32 == 0 and N % 32 == 0:
        d = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=a.codes.device)
        MX.gemm_mxfp8(a, b, out=d, bias=bias)
        rows, cols = MX.mx_quantize_rc(d, fmt, colsum=colsum, accumulate=accumulate,
                                       act="gelu" if gelu else ("dgelu" if aux is not None else None), aux=aux)
        return (d if store_d else None), rows, cols
    if M % 128 == 0 and N % 128 == 0:
        return MX.gemm_mxfp8_mx_out(a, b, fmt, out, bias=bias, aux=aux, gelu=gelu, colsum=colsum,
                                    accumulate=accumulate, store_d=store_d)
    if gelu:
        act = torch.empty((M, N), dtype=torch.bfloat16, device=a.codes.device)
        d = MX.gemm_mxfp8(a, b, out=out, bias=bias, act=act)
        src = act
    else:
        d = MX.gemm_mxfp8(a, b, out=out, bias=bias, aux=aux)
        src = d
    rows, cols = MX.mx_quantize_rc(src, fmt, colsum=colsum, accumulate=accumulate)
    return (d if store_d else None), rows, cols


class MLPBlockFn(Function):
    """x + W2 GELU(W1 LN2(x) + b1) + b2 as one autograd node (reference
    TransformerBlock second half and FeedForward, transformer.rs:89-110,151-155);
    GELU / dGELU / bias / residual live in the GEMM epilogues and the LN backward
    adds the residual gradient."""

    @staticmethod
    def forward(ctx, x2d, ln, params, fp8=None, drop=None):
        """drop: optional (FFN-hidden dropout args, FFN-output dropout args)."""
        w1, b1, w2, b2 = params
        T, F = x2d.shape[0], w1.shape[0]
        pre = torch.empty((T, F), dtype=torch.bfloat16, device=x2d.device)
        ctx.params = (ln, params)
        ctx.fp8 = fp8
        d_act, d_out = drop if drop is not None else (None, None)
        ctx.drop = (d_act, d_out)
        if _mx(fp8):
            from . import mxfp8 as MX

            gamma, beta, eps = ln
            hr, hc, mean, rstd = MX.mx_layernorm_rc(x2d, gamma.data, beta.data, eps, MX.E4M3)
            # FFN1 stores the pre-activation; GELU of it is quantised both ways (in the
            # quantiser's pass or in the GEMM's MX epilogue, as _mx_gemm_quant picks)
            with K.gemm_dropout(d_act, 2):
                _, ar, ac = _mx_gemm_quant(MX, hr, w1.mx[0], MX.E4M3, out=pre, bias=b1.data, gelu=True)
            with K.gemm_dropout(d_out, 1):
                out = MX.gemm_mxfp8(ar, w2.mx[0], bias=b2.data, residual=x2d)
            ctx.save_for_backward(x2d, mean, rstd, hc.codes, hc.sf, pre, ac.codes, ac.sf)
            return out
        if fp8 is not None:
            st, tag = fp8
            gamma, beta, eps = ln
            h8, ih, mean, rstd = st.layernorm_quantize(x2d, gamma.data, beta.data, eps, tag + ".ffn1_in", F8.E4M3)
            slot = st.epilogue_slot(tag + ".ffn2_in", F8.E4M3) if T >= 256 else None
            if slot is not None:
                # the FFN1 epilogue writes GELU straight as the FFN2 input's E4M3 codes
                a8 = torch.empty((T, F), dtype=torch.uint8, device=x2d.device)
                with K.gemm_dropout(d_act, 2):
                    F8.gemm_fp8_gelu8(h8, F8.E4M3, w1.w8, F8.E4M3, pre, a8, slot[0], slot[1], F8.E4M3,
                                      bias=b1.data, alpha=ih, alpha2=w1.w8_inv)
                ia = slot[2]
            else:
                act = torch.empty_like(pre)
                with K.gemm_dropout(d_act, 2):
                    F8.gemm_fp8(h8, F8.E4M3, w1.w8, F8.E4M3, out=pre, bias=b1.data, act=act, alpha=ih,
                                alpha2=w1.w8_inv)
                a8, ia = st.quantize(act, tag + ".ffn2_in", F8.E4M3)
            with K.gemm_dropout(d_out, 1):
                out = F8.gemm_fp8(a8, F8.E4M3, w2.w8, F8.E4M3, bias=b2.data, residual=x2d, alpha=ia,
                                  alpha2=w2.w8_inv)
            h, act = h8, a8
            ctx.inv = (ih, ia)
        else:
            h, mean, rstd = _ln_fwd(x2d, ln)
            act = torch.empty_like(pre)
            with K.gemm_dropout(d_act, 2):
                K.gemm(h, w1.w16, out=pre, bias=b1.data, act=act)
            with K.gemm_dropout(d_out, 1):
                out = K.gemm(act, w2.w16, bias=b2.data, residual=x2d)
        ctx.save_for_backward(x2d, mean, rstd, h, pre, act)
        return out

    @staticmethod
    def backward(ctx, dout):
        if _mx(ctx.fp8):
            return MLPBlockFn._backward_mx(ctx, dout)
        x2d, mean, rstd, h, pre, act = ctx.saved_tensors
        ln, (w1, b1, w2, b2) = ctx.params
        dout = dout.contiguous()
        acc = FusedGradState.accumulate
        fp8 = ctx.fp8
        d_act, d_out = ctx.drop
        dbr = K.dropout_apply(dout, d_out) if d_out is not None else dout
        if fp8 is not None:
            st, tag = fp8
            ih, ia = ctx.inv
            g8, ig = st.quantize_colsum(dbr, tag + ".ffn2_grad", F8.E5M2, b2.main_grad, acc)
            with K.gemm_dropout(d_act, 3):  # the hidden dropout's mask, then dGELU
                dpre = F8.gemm_fp8(g8, F8.E5M2, w2.w8, F8.E4M3, b_mn=True, aux=pre, alpha=ig, alpha2=w2.w8_inv)
            F8.gemm_fp8(g8, F8.E5M2, act, F8.E4M3, out=w2.main_grad, a_mn=True, b_mn=True, accumulate=acc,
                        alpha=ig, alpha2=ia)
        else:
            with K.gemm_dropout(d_act, 3):
                dpre = K.gemm(dbr, w2.w16, b_mn=True, aux=pre)
            K.gemm(dbr, act, out=w2.main_grad, a_mn=True, b_mn=True, accumulate=acc)
            K.colsum_(dbr, b2.main_grad, acc)
        _grads_done(w2, b2)
        if fp8 is not None:
            p8, ip = st.quantize_colsum(dpre, tag + ".ffn1_grad", F8.E5M2, b1.main_grad, acc)
            F8.gemm_fp8(p8, F8.E5M2, h, F8.E4M3, out=w1.main_grad, a_mn=True, b_mn=True, accumulate=acc,
                        alpha=ip, alpha2=ih)
            dh = F8.gemm_fp8(p8, F8.E5M2, w1.w8, F8.E4M3, b_mn=True, alpha=ip, alpha2=w1.w8_inv)
        else:
            K.colsum_(dpre, b1.main_grad, acc)
            K.gemm(dpre, h, out=w1.main_grad, a_mn=True, b_mn=True, accumulate=acc)
            dh = K.gemm(dpre, w1.w16, b_mn=True)
        _grads_done(w1, b1)
        return _ln_bwd(dh, x2d, mean, rstd, ln, dout), None, None, None, None

    @staticmethod
    def _backward_mx(ctx, dout):
        from . import mxfp8 as MX

        x2d, mean, rstd, hcc, hcs, pre, acc_codes, acs = ctx.saved_tensors
        ln, (w1, b1, w2, b2) = ctx.params
        dout = dout.contiguous()
        acc = FusedGradState.accumulate
        d_act, d_out = ctx.drop
        dbr = K.dropout_apply(dout, d_out) if d_out is not None else dout
        hc, ac = _mx_t(hcc, hcs, MX.E4M3), _mx_t(acc_codes, acs, MX.E4M3)
        grow, gcol = MX.mx_quantize_rc(dbr, MX.E5M2, colsum=b2.main_grad, accumulate=acc)
        # dgrad: hidden-dropout mask, then dGELU; the result is quantised both ways and its
        # columns summed into the FFN1 bias gradient (quantiser pass or MX epilogue)
        with K.gemm_dropout(d_act, 3):
            _, prow, pcol = _mx_gemm_quant(MX, grow, w2.mx[1], MX.E5M2, aux=pre, colsum=b1.main_grad,
                                           accumulate=acc, store_d=False)
        MX.gemm_mxfp8(gcol, ac, out=w2.main_grad, accumulate=acc)
        _grads_done(w2, b2)
        MX.gemm_mxfp8(pcol, hc, out=w1.main_grad, accumulate=acc)
        dh = MX.gemm_mxfp8(prow, w1.mx[1])
        _grads_done(w1, b1)
        return _ln_bwd(dh, x2d, mean, rstd, ln, dout), None, None, None, None


class EmbeddingFn(Function):
    """x = wte[ids] + wpe[pos] (reference model.rs:113-118)."""

    @staticmethod
    def forward(ctx, ids, anchor, params, seq_len, drop=None):
        wte, wpe = params
        x = K.embed_fwd(ids.reshape(-1), wte.w16, wpe.w16, seq_len, drop)
        ctx.save_for_backward(ids)
        ctx.params = params
        ctx.seq_len = seq_len
        ctx.drop = drop
        return x

    @staticmethod
    def backward(ctx, dx):
        (ids,) = ctx.saved_tensors
        wte, wpe = ctx.params
        if ctx.drop is not None:
            dx = K.dropout_apply(dx.contiguous(), ctx.drop)
        K.embed_bwd(ids.reshape(-1), dx, wte.main_grad, wpe.main_grad, ctx.seq_len,
                    FusedGradState.accumulate)
        _grads_done(wte, wpe)
        return None, None, None, None, None


class LMHeadLossFn(Function):
    """mean CE(lm_head(h), targets) with dlogits computed in the forward kernel
    (reference cross_entropy_loss, examples/gpt-1b/src/main.rs:32-41).

    grad_scale (device fp32 scalar, optional) multiplies the gradients, e.g. the
    dynamic loss scale; the returned loss is unscaled.  fp8 (an ``Fp8State``,
    optional): the three LM-head GEMMs run in FP8 with per-tensor delayed scaling --
    h and the weight as E4M3, dlogits as E5M2 -- instead of bf16."""

    @staticmethod
    def forward(ctx, h, targets, params, grad_scale, fp8=None):
        w, b = params
        T = h.shape[0]
        ctx.fp8 = fp8
        ctx.g8 = False
        if fp8 is not None:
            h8, ih = fp8.quantize(h, "lm_head.in", F8.E4M3)
            logits = F8.gemm_fp8(h8, F8.E4M3, w.w8, F8.E4M3, bias=b.data, alpha=ih, alpha2=w.w8_inv)
            slot = fp8.epilogue_slot("lm_head.grad", F8.E5M2)
            if slot is not None:
                # the cross-entropy kernel writes dlogits straight as the backward GEMMs' E5M2
                # operand (the delayed scale is known), so no bf16 dlogits and no quantise pass
                g8 = torch.empty(logits.shape, dtype=torch.uint8, device=logits.device)
                rows = K.xent_fused(logits, targets.reshape(-1), grad_scale, 1.0 / T, True, out8=g8,
                                    out8_scale=slot[0], out8_amax=slot[1])
                ctx.g8 = True
                ctx.save_for_backward(h8, ih, g8, slot[2])
                ctx.params = params
                return rows.mean()
            saved = (h8, ih)
        else:
            logits = K.gemm(h, w.w16, bias=b.data)
            saved = (h,)
        rows = K.xent_fused(logits, targets.reshape(-1), grad_scale, 1.0 / T, True)
        ctx.save_for_backward(*saved, logits)
        ctx.params = params
        return rows.mean()

    @staticmethod
    def backward(ctx, gloss):
        w, b = ctx.params
        acc = FusedGradState.accumulate
        g = gloss.reshape(1).float().contiguous()
        if ctx.fp8 is not None:
            if ctx.g8:
                h8, ih, g8, igd = ctx.saved_tensors
                K.colsum_e5m2_(g8, b.main_grad, acc, scale=igd, scale2=g)  # bias gradient from the codes
            else:
                h8, ih, dlogits = ctx.saved_tensors
                g8, igd = ctx.fp8.quantize(dlogits, "lm_head.grad", F8.E5M2)
                K.colsum_(dlogits, b.main_grad, acc, scale=g)
            a = igd * g  # the E5M2 inverse scale times the incoming loss gradient
            dh = F8.gemm_fp8(g8, F8.E5M2, w.w8, F8.E4M3, b_mn=True, alpha=a, alpha2=w.w8_inv)
            F8.gemm_fp8(g8, F8.E5M2, h8, F8.E4M3, out=w.main_grad, a_mn=True, b_mn=True, accumulate=acc,
                        alpha=a, alpha2=ih, out_dtype=torch.float32)
        else:
            h, dlogits = ctx.saved_tensors
            dh = K.gemm(dlogits, w.w16, b_mn=True, alpha=g)
            K.gemm(dlogits, h, out=w.main_grad, a_mn=True, b_mn=True, accumulate=acc, alpha=g)
            K.colsum_(dlogits, b.main_grad, acc, scale=g)
        _grads_done(w, b)
        return dh, None, None, None, None
