"""Causal multi-head attention for the fused GPT path (sm_100a flash attention).

Reference: scores = QK^T / sqrt(d_head) + mask -> softmax -> dropout -> PV
(examples/gpt-1b/src/transformer.rs:51-85) with the [S,S] 0/-inf causal mask
(transformer.rs:163-171).  The mask is applied by index inside the kernels and
the [B,H,S,S] score tensor is never materialised: ``csrc/kernels/attention.cu``
runs the forward (O and the per-row log-sum-exp) and the backward (dQ, dK, dV
straight into one [T, 3*H*d] gradient matrix) on tcgen05 with TMEM
accumulators.  Head dim 128 and sequence lengths that are multiples of 128.
Attention-probability dropout (``drop``) draws its Philox mask inside both
kernels (``csrc/kernels/philox.cuh``): element (q, k) of head (b, h) is element
((b*H + h) * S + q) * S + k of the site.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .._ext import cuda as _cuda

HEAD_DIM = 128
TILE = 128


def check_shape(S: int, dh: int) -> None:
    if dh != HEAD_DIM or S % TILE != 0:
        raise ValueError(f"fused attention needs head dim {HEAD_DIM} and seq len % {TILE} == 0 "
                         f"(got head dim {dh}, seq len {S})")


def attention_fwd(qkv: torch.Tensor, B: int, S: int, H: int, drop=None, mx_fmt: Optional[int] = None):
    """qkv [B*S, 3*H*128] bf16 -> (out [B*S, H*128] bf16, lse [B, H, S] fp32).
    drop: optional (rng, site, thr16, scale) of the attention-probability dropout.
    mx_fmt (optional MXFP8 format): the epilogue also writes the output's MXFP8 row and
    column codes (what ``mx_quantize_rc`` makes of ``out``) and the call returns
    (out, lse, rows, cols)."""
    kw = {}
    rows = cols = None
    if mx_fmt is not None:
        from .mxfp8 import MX_FMT_MAX, MxTensor, sf_numel

        T, HD = B * S, H * 128
        dev = qkv.device
        rows = MxTensor(torch.empty((T, HD), dtype=torch.uint8, device=dev),
                        torch.empty(sf_numel(T, HD), dtype=torch.uint8, device=dev), int(mx_fmt))
        cols = MxTensor(torch.empty((HD, T), dtype=torch.uint8, device=dev),
                        torch.empty(sf_numel(HD, T), dtype=torch.uint8, device=dev), int(mx_fmt))
        kw = dict(mx_rc=rows.codes, mx_rsf=rows.sf, mx_cc=cols.codes, mx_csf=cols.sf, mx_fmt=int(mx_fmt),
                  mx_fmax=float(MX_FMT_MAX[mx_fmt]))
    if drop is None:
        out, lse = _cuda().attn_fwd(qkv, B, S, H, **kw)
    else:
        rng, site, thr, scale = drop
        out, lse = _cuda().attn_fwd(qkv, B, S, H, rng, int(site), int(thr), float(scale), **kw)
    return (out, lse) if mx_fmt is None else (out, lse, rows, cols)


def attention_bwd(dout: torch.Tensor, qkv: torch.Tensor, out: torch.Tensor, lse: torch.Tensor,
                  B: int, S: int, H: int, drop=None, dq_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """-> dqkv [B*S, 3*H*128] bf16 (dq | dk | dv).  With dq_out (fp32 [B*S, H*128]) dQ is
    left there in fp32 and the dq third of dqkv is not written."""
    if drop is None:
        return _cuda().attn_bwd(dout.contiguous(), qkv, out, lse, B, S, H, dq_out=dq_out)
    rng, site, thr, scale = drop
    return _cuda().attn_bwd(dout.contiguous(), qkv, out, lse, B, S, H, rng, int(site), int(thr), float(scale),
                            dq_out=dq_out)


class CausalAttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, B, S, H):
        out, lse = attention_fwd(qkv, B, S, H)
        ctx.save_for_backward(qkv, out, lse)
        ctx.dims = (B, S, H)
        return out

    @staticmethod
    def backward(ctx, dout):
        qkv, out, lse = ctx.saved_tensors
        return attention_bwd(dout, qkv, out, lse, *ctx.dims), None, None, None


def causal_attention(qkv: torch.Tensor, B: int, S: int, H: int, dh: int) -> torch.Tensor:
    """qkv: [B*S, 3*H*dh] bf16 (q | k | v, heads contiguous) -> [B*S, H*dh]."""
    check_shape(S, dh)
    return CausalAttentionFn.apply(qkv, B, S, H)


def reference_attention(qkv: torch.Tensor, B: int, S: int, H: int, dh: int,
                        keep: torch.Tensor = None, p_drop: float = 0.0) -> torch.Tensor:
    """Plain PyTorch fp32 oracle of the same op (tests only); keep: optional bool
    [B, H, S, S] dropout mask of the probabilities."""
    q, k, v = qkv.float().view(B, S, 3, H, dh).unbind(2)
    q, k, v = (t.transpose(1, 2) for t in (q, k, v))
    s = q @ k.transpose(-1, -2) / dh ** 0.5
    mask = torch.ones(S, S, dtype=torch.bool, device=qkv.device).triu(1)
    p = torch.softmax(s.masked_fill(mask, float("-inf")), dim=-1)
    if keep is not None:
        p = torch.where(keep, p / (1.0 - p_drop), torch.zeros_like(p))
    return (p @ v).transpose(1, 2).reshape(B * S, H * dh)
