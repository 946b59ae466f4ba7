"""Causal multi-head attention for the fused GPT path.

Reference: scores = QK^T / sqrt(d_head) + mask -> softmax -> dropout -> PV
(examples/gpt-1b/src/transformer.rs:51-85) with the [S,S] 0/-inf causal mask
(transformer.rs:163-171).  The mask is applied by index here (no mask tensor)
and the [B,H,S,S] score tensor is never materialised.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def causal_attention(qkv: torch.Tensor, B: int, S: int, H: int, dh: int) -> torch.Tensor:
    """qkv: [B*S, 3*H*dh] bf16 (q | k | v, heads contiguous) -> [B*S, H*dh]."""
    q, k, v = qkv.view(B, S, 3, H, dh).unbind(2)
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                       is_causal=True)
    return o.transpose(1, 2).reshape(B * S, H * dh)
