"""Thin Python wrappers over the sm_100a kernels of ``mtorus._cuda``.

Each wrapper allocates outputs with torch's caching allocator and launches on
the current stream.  None of them falls back to eager PyTorch: on a CUDA tensor
the extension must be present (``mtorus._ext.cuda`` raises otherwise).
"""
from __future__ import annotations

import os
import sys
from typing import Optional

import torch

from .._ext import cuda as _cuda

_TRACE = bool(os.environ.get("MTORUS_TRACE"))


def layernorm_fwd(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5):
    """bf16 LayerNorm over the last dim with fp32 gamma/beta -> (y, mean, rstd)."""
    return _cuda().layernorm_fwd(x.contiguous(), gamma, beta, float(eps))


def layernorm_bwd(dy, x, gamma, mean, rstd, dgamma, dbeta, accumulate: bool, dres=None):
    """Returns dx (+ dres, the gradient arriving through a residual branch that
    reads x); writes (accumulate=False) or adds dgamma/dbeta (fp32)."""
    return _cuda().layernorm_bwd(dy.contiguous(), x, gamma, mean, rstd, dgamma, dbeta, bool(accumulate),
                                 None if dres is None else dres.contiguous())


def xent_fused(logits: torch.Tensor, targets: torch.Tensor, grad_scale: Optional[torch.Tensor] = None,
               scale_mul: float = 1.0, write_grad: bool = True, out8: Optional[torch.Tensor] = None,
               out8_scale: Optional[torch.Tensor] = None, out8_amax: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-row CE loss; when write_grad, logits are overwritten in place with
    grad_scale * scale_mul * (softmax - onehot) -- or, with out8 (uint8 like the logits),
    those dlogits are written there as E5M2 codes times out8_scale (the logits stay) and
    their max |value| goes into out8_amax."""
    return _cuda().xent_fused(logits, targets, grad_scale, float(scale_mul), bool(write_grad), out8=out8,
                              out8_scale=out8_scale, out8_amax=out8_amax)


def gemm(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None, *, a_mn: bool = False,
         b_mn: bool = False, bias=None, residual=None, act=None, aux=None, alpha=None,
         accumulate: bool = False, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """tcgen05 GEMM: out[M,N] = epilogue(alpha * A . B^T).

    A is [M,K] (or [K,M] with a_mn=True), B is [N,K] (or [K,N] with b_mn=True).
    Epilogue: + bias[N] (fp32), + residual[M,N], act <- GELU(out) (out keeps the
    pre-activation), out *= GELU'(aux) (dGELU), fp32 out with accumulate adds into out.
    """
    M = a.shape[1] if a_mn else a.shape[0]
    N = b.shape[1] if b_mn else b.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    if _TRACE:
        print(f"[gemm] A{tuple(a.shape)}{tuple(a.stride())} a_mn={a_mn} B{tuple(b.shape)}{tuple(b.stride())} "
              f"b_mn={b_mn} out{tuple(out.shape)} {out.dtype} bias={bias is not None} res={residual is not None} "
              f"act={act is not None} aux={aux is not None} alpha={alpha is not None} acc={accumulate}",
              file=sys.stderr, flush=True)
    _cuda().gemm_bf16(a, bool(a_mn), b, bool(b_mn), out, bias, residual, act, aux, alpha, bool(accumulate))
    return out


def gemm_status(reset: bool = True) -> int:
    """Non-zero when a GEMM launch timed out on an internal wait (status code of the role)."""
    return int(_cuda().gemm_status(reset))


def embed_fwd(ids, wte16, wpe16, seq_len: int, drop=None):
    """drop: optional (rng, site, thr16, scale) of the embedding dropout (``DropoutState.args``)."""
    if drop is None:
        return _cuda().embed_fwd(ids, wte16, wpe16, int(seq_len))
    rng, site, thr, scale = drop
    return _cuda().embed_fwd(ids, wte16, wpe16, int(seq_len), rng, int(site), int(thr), float(scale))


def dropout_apply(x, drop, out=None):
    """x * keep * scale with the site's Philox mask (the backward of a dropout); bf16."""
    rng, site, thr, scale = drop
    x = x.contiguous()
    if out is None:
        out = torch.empty_like(x)
    _cuda().dropout_apply(x, out, rng, int(site), int(thr), float(scale))
    return out


def _lib_carveout_default() -> bool:
    import os

    return os.environ.get("MTORUS_DP_LIB_CARVEOUT", "1") != "0"


LIB_CARVEOUT = _lib_carveout_default()


def set_reserved_sms(n: int) -> None:
    """Keep ``n`` SMs out of the GEMM grids launched from now on, for kernels that overlap
    them on another stream (the data-parallel reduce-scatter during backward): the own GEMM
    kernels size their grids without those SMs, and the library GEMMs get the same count as
    torch's cuBLASLt SM carveout (``MTORUS_DP_LIB_CARVEOUT=0`` leaves the library GEMMs on every
    SM).  ``n = 0`` releases both."""
    _cuda().gemm_set_reserved_sms(int(n))
    if LIB_CARVEOUT and hasattr(torch._C, "_set_sm_carveout_experimental"):
        import warnings

        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            torch._C._set_sm_carveout_experimental(int(n) if n else None)


class gemm_dropout:
    """``with gemm_dropout(drop, mode): <one GEMM call>`` -- dropout drawn in that GEMM's
    epilogue (drop = (rng, site, thr16, scale) or None for none): mode 1 drops the result
    before the residual add, 2 drops the GELU output, 3 masks the incoming gradient before
    the dGELU.  The setting is consumed by the next GEMM launch and cleared on exit in
    any case, so it never leaks into a later GEMM."""

    armed = False  # a setting is pending: the GEMM inside must be this library's kernel

    def __init__(self, drop, mode: int):
        self.drop, self.mode = drop, mode

    def __enter__(self):
        if self.drop is not None:
            rng, site, thr, scale = self.drop
            _cuda().gemm_set_dropout(rng, int(site), int(thr), float(scale), int(self.mode))
            gemm_dropout.armed = True
        return self

    def __exit__(self, *exc):
        if self.drop is not None:
            _cuda().gemm_set_dropout(None, 0, 0, 1.0, 0)
            gemm_dropout.armed = False
        return False


def embed_bwd(ids, dy, dwte, dwpe, seq_len: int, accumulate: bool):
    _cuda().embed_bwd(ids, dy.contiguous(), dwte, dwpe, int(seq_len), bool(accumulate))


def bias_gelu_fwd(pre, bias=None):
    return _cuda().bias_gelu_fwd(pre, bias)


def gelu_bwd_(dact, pre):
    _cuda().gelu_bwd_(dact, pre)
    return dact


def colsum_(x, out, accumulate: bool, scale=None):
    """out (+)= scale * column sums of x (bf16 [rows, F] -> fp32 [F])."""
    _cuda().colsum_(x.contiguous(), out, bool(accumulate), scale)
    return out


def colsum_e5m2_(codes, out, accumulate: bool, scale=None, scale2=None):
    """out (+)= scale * scale2 * column sums of E5M2 codes (uint8 [rows, F] -> fp32 [F])."""
    _cuda().colsum_e5m2_(codes.contiguous(), out, bool(accumulate), scale, scale2)
    return out


def grad_sumsq(g, state):
    _cuda().optim_grad_sumsq(g, state)


def optim_finalize(state, dynamic: bool, growth_interval: int, max_norm: float, unscale: bool = True):
    _cuda().optim_finalize(state, bool(dynamic), int(growth_interval), float(max_norm), bool(unscale))


def adam_step(p, m, v, g, w16, state, lr, beta1=0.9, beta2=0.999, eps=1e-5, weight_decay=0.0, step_override=0.0):
    _cuda().adam_step(p, m, v, g, w16, state, float(lr), float(beta1), float(beta2), float(eps),
                      float(weight_decay), float(step_override))


def sgd_step(p, g, w16, state, lr):
    _cuda().sgd_step(p, g, w16, state, float(lr))
