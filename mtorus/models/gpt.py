"""GPT decoder (the reference's example model) with a fused sm_100a fast path.

Module tree and parameter names follow the reference GPT example
(examples/gpt-1b/src/model.rs:56-129, transformer.rs:12-171):

    token_embedding, position_embedding, blocks.{i}.{attention.{q,k,v,out}_proj,
    ff.linear{1,2}, norm{1,2}}, ln_f, lm_head

Linear weights use torch's [out, in] convention; LayerNorm parameters are named
``gamma`` / ``beta`` as in Burn.

Two execution paths share the same parameters:

* ``forward(input_ids)`` -- the reference semantics in plain PyTorch ops (any
  device / dtype): learned positions, additive 0/-inf causal mask, softmax
  attention, erf-GELU, dropout.  This is the CPU oracle.
* ``fused_loss(input_ids, targets)`` -- the B200 path: bf16 activations, every
  Linear on the tcgen05 GEMM with bias / GELU / residual / dGELU fused in the
  epilogue, fused LayerNorm, embedding and cross-entropy kernels, gradients
  written straight into the flat fp32 ``main_grad`` buffer.  Requires the model
  to be flattened with ``flatten()``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class GptConfig:
    """Reference: GptConfig (examples/gpt-1b/src/model.rs:12-49)."""

    vocab_size: int
    d_model: int
    num_layers: int
    num_heads: int
    d_ff: int
    max_seq_len: int
    dropout: float = 0.1

    @staticmethod
    def gpt_1b() -> "GptConfig":
        """The reference's ~1B configuration (model.rs:25-37)."""
        return GptConfig(50257, 2048, 24, 32, 8192, 2048, 0.1)

    @staticmethod
    def test_config() -> "GptConfig":
        """The reference's small CPU configuration (model.rs:39-49)."""
        return GptConfig(1000, 128, 2, 4, 512, 64, 0.1)

    @staticmethod
    def gpt_1b_bench() -> "GptConfig":
        """GPT-1B training benchmark shape: 24 layers, d 2048, 16 heads, d_ff 8192,
        vocab 50304, seq 2048 (dropout off)."""
        return GptConfig(50304, 2048, 24, 16, 8192, 2048, 0.0)

    @staticmethod
    def gpt_6_7b() -> "GptConfig":
        """GPT-3 style 6.7B: 32 layers, d 4096, 32 heads, d_ff 16384, vocab 50304."""
        return GptConfig(50304, 4096, 32, 32, 16384, 2048, 0.0)

    @staticmethod
    def example_tiny() -> "GptConfig":
        """Tiny CPU example: 2 layers, d 128, 4 heads, d_ff 512, vocab 1024, seq 64."""
        return GptConfig(1024, 128, 2, 4, 512, 64, 0.1)

    def num_params(self) -> int:
        d, f, V, S, L = self.d_model, self.d_ff, self.vocab_size, self.max_seq_len, self.num_layers
        block = 4 * (d * d + d) + (d * f + f) + (f * d + d) + 4 * d
        return V * d + S * d + L * block + 2 * d + (d * V + V)

    def train_flops_per_token(self, seq_len: Optional[int] = None) -> float:
        """6 x GEMM parameters + causal attention (fwd+bwd), per token."""
        S = seq_len or self.max_seq_len
        d, f, V, L = self.d_model, self.d_ff, self.vocab_size, self.num_layers
        gemm = L * (4 * d * d + 2 * d * f) + d * V
        attn = L * 2 * 2 * S * d * 0.5  # QK^T and PV, causal half
        return 6.0 * gemm + 3.0 * attn


class LayerNorm(nn.Module):
    def __init__(self, d: int, eps: float = 1e-5):
        super().__init__()
        self.gamma = nn.Parameter(torch.ones(d))
        self.beta = nn.Parameter(torch.zeros(d))
        self.eps = eps

    def forward(self, x):
        return F.layer_norm(x, (x.shape[-1],), self.gamma.to(x.dtype), self.beta.to(x.dtype), self.eps)


class Linear(nn.Module):
    def __init__(self, d_in: int, d_out: int, bias: bool = True):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(d_out, d_in))
        self.bias = nn.Parameter(torch.empty(d_out)) if bias else None
        bound = 1.0 / math.sqrt(d_in)
        nn.init.uniform_(self.weight, -bound, bound)
        if self.bias is not None:
            nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, x):
        return F.linear(x, self.weight.to(x.dtype), None if self.bias is None else self.bias.to(x.dtype))


class Embedding(nn.Module):
    def __init__(self, n: int, d: int):
        super().__init__()
        self.weight = nn.Parameter(torch.randn(n, d))

    def forward(self, ids):
        return F.embedding(ids, self.weight)


def create_causal_mask(seq_len: int, device=None, dtype=torch.float32) -> torch.Tensor:
    """[S, S] additive mask: 0 on and below the diagonal, -inf above
    (reference create_causal_mask, transformer.rs:163-171)."""
    m = torch.zeros(seq_len, seq_len, device=device, dtype=dtype)
    return m.masked_fill(torch.ones(seq_len, seq_len, dtype=torch.bool, device=device).triu(1), float("-inf"))


def create_position_ids(batch_size: int, seq_len: int, device=None) -> torch.Tensor:
    return torch.arange(seq_len, device=device).unsqueeze(0).expand(batch_size, seq_len)


class _ParamView:
    """A contiguous run of flat-buffer parameters seen as one matrix/vector."""

    def __init__(self, members, flat, shape):
        self.members = members
        self.data = flat.contiguous_view(members, "master").view(shape)
        self.w16 = flat.contiguous_view(members, "w16").view(shape)
        self.main_grad = flat.contiguous_view(members, "grad").view(shape)
        self.shape = shape


class MultiHeadAttention(nn.Module):
    def __init__(self, d_model: int, num_heads: int, dropout: float = 0.1):
        super().__init__()
        assert d_model % num_heads == 0, f"d_model ({d_model}) must be divisible by num_heads ({num_heads})"
        self.q_proj = Linear(d_model, d_model)
        self.k_proj = Linear(d_model, d_model)
        self.v_proj = Linear(d_model, d_model)
        self.out_proj = Linear(d_model, d_model)
        self.dropout = nn.Dropout(dropout)
        self.num_heads = num_heads
        self.d_head = d_model // num_heads
        self.d_model = d_model

    def forward(self, x, mask: Optional[torch.Tensor] = None):
        B, S, _ = x.shape
        q = self.q_proj(x).reshape(B, S, self.num_heads, self.d_head).transpose(1, 2)
        k = self.k_proj(x).reshape(B, S, self.num_heads, self.d_head).transpose(1, 2)
        v = self.v_proj(x).reshape(B, S, self.num_heads, self.d_head).transpose(1, 2)
        scores = q.matmul(k.transpose(2, 3)) * (1.0 / math.sqrt(self.d_head))
        if mask is not None:
            scores = scores + mask.to(scores.dtype)
        attn = self.dropout(torch.softmax(scores, dim=3))
        out = attn.matmul(v).transpose(1, 2).reshape(B, S, self.d_model)
        return self.out_proj(out)


class FeedForward(nn.Module):
    def __init__(self, d_model: int, d_ff: int, dropout: float = 0.1):
        super().__init__()
        self.linear1 = Linear(d_model, d_ff)
        self.linear2 = Linear(d_ff, d_model)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x):
        return self.linear2(self.dropout(F.gelu(self.linear1(x))))


class TransformerBlock(nn.Module):
    def __init__(self, d_model: int, num_heads: int, d_ff: int, dropout: float = 0.1):
        super().__init__()
        self.attention = MultiHeadAttention(d_model, num_heads, dropout)
        self.ff = FeedForward(d_model, d_ff, dropout)
        self.norm1 = LayerNorm(d_model)
        self.norm2 = LayerNorm(d_model)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x, mask: Optional[torch.Tensor] = None):
        x = self.dropout(self.attention(self.norm1(x), mask)) + x
        return self.dropout(self.ff(self.norm2(x))) + x

    # ---------------------------------------------------------------- fused path
    def fused_forward(self, x2d, B: int, S: int, fp8=None, drop=None):
        """drop: optional (DropoutState, layer index) -- the layer's four dropout sites
        (attention probabilities, attention output, FFN hidden, FFN output) drawn in the
        producing kernels."""
        from ..ops.dropout import SITE_ATTN_OUT, SITE_ATTN_PROBS, SITE_FFN_ACT, SITE_FFN_OUT
        from ..ops.fused import AttnBlockFn, MLPBlockFn

        a = self.attention
        da = dm = None
        if drop is not None:
            st, layer = drop
            da = (st.layer_args(layer, SITE_ATTN_PROBS), st.layer_args(layer, SITE_ATTN_OUT))
            dm = (st.layer_args(layer, SITE_FFN_ACT), st.layer_args(layer, SITE_FFN_OUT))
        x2d = AttnBlockFn.apply(x2d, (self.norm1.gamma, self.norm1.beta, self.norm1.eps),
                                (self._qkv_w, self._qkv_b), (a.out_proj.weight, a.out_proj.bias),
                                (B, S, a.num_heads, a.d_head), fp8, da)
        return MLPBlockFn.apply(x2d, (self.norm2.gamma, self.norm2.beta, self.norm2.eps),
                                (self.ff.linear1.weight, self.ff.linear1.bias,
                                 self.ff.linear2.weight, self.ff.linear2.bias), fp8, dm)


class GptModel(nn.Module):
    """Reference: GptModel (examples/gpt-1b/src/model.rs:56-129)."""

    def __init__(self, config: GptConfig, init: str = "reference", layers: Optional[Tuple[int, int]] = None,
                 embed: bool = True, head: bool = True):
        """``layers=(lo, hi)`` / ``embed`` / ``head`` build one pipeline stage: blocks
        lo..hi-1 of the full model, with the embeddings only on the first stage and
        ln_f + lm_head only on the last (the reference splits its layer list the same
        way, crates/mt-burn/src/module_ext.rs:40-79)."""
        super().__init__()
        c = config
        self.config = c
        lo, hi = layers if layers is not None else (0, c.num_layers)
        self.layer_offset = lo
        self.has_embed, self.has_head = embed, head
        if embed:
            self.token_embedding = Embedding(c.vocab_size, c.d_model)
            self.position_embedding = Embedding(c.max_seq_len, c.d_model)
        self.blocks = nn.ModuleList(
            [TransformerBlock(c.d_model, c.num_heads, c.d_ff, c.dropout) for _ in range(lo, hi)])
        if head:
            self.ln_f = LayerNorm(c.d_model)
            self.lm_head = Linear(c.d_model, c.vocab_size)
        self.dropout = nn.Dropout(c.dropout)
        self.d_model = c.d_model
        self.max_seq_len = c.max_seq_len
        self.vocab_size = c.vocab_size
        self.flat = None
        if init == "normal":
            self.init_normal_(0.02)

    @torch.no_grad()
    def init_normal_(self, std: float = 0.02, generator: Optional[torch.Generator] = None):
        """N(0, std) weights, zero biases, unit LayerNorm gains."""
        for name, p in self.named_parameters():
            if name.endswith("gamma"):
                p.fill_(1.0)
            elif name.endswith("beta") or name.endswith("bias"):
                p.zero_()
            else:
                p.normal_(0.0, std, generator=generator)

    def num_layers(self) -> int:
        return len(self.blocks)

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        return self.forward_stage(input_ids)

    def forward_stage(self, x: torch.Tensor) -> torch.Tensor:
        """Reference path of a (possibly partial) model: token ids [B, S] on the first
        stage, else the previous stage's [B, S, d] hidden; returns the hidden, or the
        logits when this part holds the head."""
        if self.has_embed:
            B, S = x.shape
            dev = x.device
            hidden = self.token_embedding(x) + self.position_embedding(create_position_ids(B, S, dev))
            hidden = self.dropout(hidden)
        else:
            hidden, S, dev = x, x.shape[1], x.device
        mask = create_causal_mask(S, dev).reshape(1, 1, S, S)
        for blk in self.blocks:
            hidden = blk(hidden, mask)
        if self.has_head:
            return self.lm_head(self.ln_f(hidden))
        return hidden

    # ---------------------------------------------------------------- fused path
    def flat_groups(self) -> List[List[nn.Parameter]]:
        """Parameter layout for the flat buffers: q/k/v weights (and biases) back to back."""
        groups = [[self.token_embedding.weight], [self.position_embedding.weight]] if self.has_embed else []
        for blk in self.blocks:
            a = blk.attention
            groups += [[blk.norm1.gamma, blk.norm1.beta],
                       [a.q_proj.weight, a.k_proj.weight, a.v_proj.weight],
                       [a.q_proj.bias, a.k_proj.bias, a.v_proj.bias],
                       [a.out_proj.weight], [a.out_proj.bias],
                       [blk.norm2.gamma, blk.norm2.beta],
                       [blk.ff.linear1.weight], [blk.ff.linear1.bias],
                       [blk.ff.linear2.weight], [blk.ff.linear2.bias]]
        if self.has_head:
            groups += [[self.ln_f.gamma, self.ln_f.beta], [self.lm_head.weight], [self.lm_head.bias]]
        return groups

    def flatten(self, device, grad_dtype=torch.float32, symmetric: bool = False, group=None):
        """Move parameters into flat fp32/bf16/grad buffers on `device` (fused path);
        ``symmetric`` places gradients and bf16 weights in peer-mapped memory for
        the fused NVLink data-parallel path."""
        from ..parallel.flat import FlatParams

        self.flat = FlatParams(self.flat_groups(), device, grad_dtype=grad_dtype, symmetric=symmetric, group=group)
        d = self.d_model
        for blk in self.blocks:
            a = blk.attention
            blk._qkv_w = _ParamView([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], self.flat, (3 * d, d))
            blk._qkv_b = _ParamView([a.q_proj.bias, a.k_proj.bias, a.v_proj.bias], self.flat, (3 * d,))
        return self.flat

    def fused_hidden(self, input_ids: torch.Tensor) -> torch.Tensor:
        from ..ops.fused import LayerNormFn

        assert self.flat is not None, "call flatten(device) before using the fused path"
        B, S = input_ids.shape
        x = self.fused_blocks(self.fused_embed(input_ids), B, S)
        return LayerNormFn.apply(x, (self.ln_f.gamma, self.ln_f.beta), self.ln_f.eps)

    def fused_embed(self, input_ids: torch.Tensor) -> torch.Tensor:
        """[B, S] token ids -> [B*S, d] bf16 hidden (token + learned position embedding,
        then the embedding dropout when enabled)."""
        from ..ops.dropout import SITE_EMBED
        from ..ops.fused import EmbeddingFn, grad_anchor

        assert self.flat is not None, "call flatten(device) before using the fused path"
        S = input_ids.shape[1]
        ds = self.dropout_state
        return EmbeddingFn.apply(input_ids, grad_anchor(input_ids.device),
                                 (self.token_embedding.weight, self.position_embedding.weight), S,
                                 None if ds is None else ds.args(SITE_EMBED))

    dropout_state = None

    def enable_dropout(self, seed: int = 0):
        """Dropout with the config's probability in the fused path (all five reference
        sites, masks drawn by Philox inside the kernels); no-op for p = 0.  The trainer
        calls ``dropout_state.advance()`` once per step and sets
        ``dropout_state.micro`` before each micro-batch's forward."""
        from ..ops.dropout import DropoutState

        p = float(getattr(self.config, "dropout", 0.0))
        self.dropout_state = DropoutState(p, self.flat.device, seed) if p > 0.0 else None
        return self.dropout_state

    def _layer_drop(self, i: int):
        ds = self.dropout_state
        return None if ds is None else (ds, self.layer_offset + i)

    def fused_blocks(self, x: torch.Tensor, B: int, S: int) -> torch.Tensor:
        """[B*S, d] -> [B*S, d] through this model's (or stage's) transformer blocks."""
        st = getattr(self, "fp8_state", None)
        for i, blk in enumerate(self.blocks):
            x = blk.fused_forward(x, B, S, None if st is None else (st, f"L{self.layer_offset + i}"),
                                  self._layer_drop(i))
        return x

    def fused_stage(self, x: torch.Tensor, B: int, S: int) -> torch.Tensor:
        """Pipeline-stage forward: token ids (first stage) or the previous stage's
        [B*S, d] hidden in, this stage's [B*S, d] hidden out (before ln_f)."""
        if self.has_embed:
            x = self.fused_embed(x)
        return self.fused_blocks(x, B, S)

    def fused_stage_segments(self, B: int, S: int) -> list:
        """``fused_stage`` as one callable per transformer block (the embedding folded
        into the first): the segments that selective activation checkpointing splits
        at the midpoint."""
        st = getattr(self, "fp8_state", None)

        def block_fn(i, blk, embed):
            def run(x):
                if embed:
                    x = self.fused_embed(x)
                return blk.fused_forward(x, B, S, None if st is None else (st, f"L{self.layer_offset + i}"),
                                         self._layer_drop(i))
            return run

        return [block_fn(i, blk, self.has_embed and i == 0) for i, blk in enumerate(self.blocks)]

    def fused_head_loss(self, x: torch.Tensor, targets: torch.Tensor,
                        grad_scale: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Last-stage loss: ln_f -> lm_head -> mean CE, gradients into main_grad."""
        from ..ops.fused import LayerNormFn, LMHeadLossFn

        h = LayerNormFn.apply(x, (self.ln_f.gamma, self.ln_f.beta), self.ln_f.eps)
        return LMHeadLossFn.apply(h, targets, (self.lm_head.weight, self.lm_head.bias), grad_scale,
                                  self._head_fp8())

    # ---------------------------------------------------------------- FP8
    def fp8_weights(self):
        """(name, weight-like) pairs of the transformer blocks' GEMMs (the block recipe;
        the LM head, when in FP8, uses per-tensor scales, see ``enable_fp8``)."""
        out = []
        for j, blk in enumerate(self.blocks):
            i = self.layer_offset + j
            out += [(f"L{i}.qkv_w", blk._qkv_w), (f"L{i}.out_w", blk.attention.out_proj.weight),
                    (f"L{i}.ffn1_w", blk.ff.linear1.weight), (f"L{i}.ffn2_w", blk.ff.linear2.weight)]
        return out

    def enable_fp8(self, history: int = 16, recipe: str = "tensor", head: bool = True):
        """E4M3 weights / activations and E5M2 gradients for the block GEMMs; call
        ``refresh_fp8_weights()`` after every optimizer step and ``fp8_state.end_step()``
        at the end of every step.  recipe "tensor": per-tensor scales with delayed
        scaling (amax histories); "mx": MXFP8, one power-of-two scale per 32 values
        along each GEMM's contraction dimension, for all three GEMMs of every block
        linear (``mtorus.ops.mxfp8``).  head: the LM head's three GEMMs in FP8 as well
        (per-tensor delayed scaling in both recipes), else bf16."""
        from ..ops.fp8 import Fp8State

        assert self.flat is not None, "flatten() first"
        if recipe not in ("tensor", "mx"):
            raise ValueError(f"fp8 recipe must be 'tensor' or 'mx', not {recipe!r}")
        self.fp8_state = Fp8State(self.flat.device, history)
        self.fp8_state.recipe = recipe
        for name, w in self.fp8_weights():
            if recipe == "tensor":
                w.w8 = torch.empty(w.shape, dtype=torch.uint8, device=self.flat.device)
            w.fp8_name = name
        self.fp8_head = bool(head) and self.has_head and self.flat.device.type == "cuda"  # per-tensor kernels
        if self.fp8_head:
            w = self.lm_head.weight
            w.w8 = torch.empty(w.shape, dtype=torch.uint8, device=self.flat.device)
        return self.fp8_state

    def refresh_fp8_weights(self):
        from ..ops import fp8 as F8

        st = self.fp8_state
        if getattr(self, "fp8_head", False):
            w = self.lm_head.weight
            _, w.w8_inv = st.quantize_into(w.w16, "lm_head.w", F8.E4M3, w.w8)
        if st.recipe == "mx":
            from ..ops.mxfp8 import E4M3, mx_quantize_rc

            for _, w in self.fp8_weights():
                w.mx = mx_quantize_rc(w.w16, E4M3)  # (row-wise: forward, column-wise: dgrad)
            return
        for name, w in self.fp8_weights():
            _, w.w8_inv = st.quantize_into(w.w16, name, F8.E4M3, w.w8)

    def fused_loss(self, input_ids: torch.Tensor, targets: torch.Tensor,
                   grad_scale: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Mean next-token CE through the fused kernels; backward writes main_grad."""
        from ..ops.fused import LMHeadLossFn

        h = self.fused_hidden(input_ids)
        return LMHeadLossFn.apply(h, targets, (self.lm_head.weight, self.lm_head.bias), grad_scale,
                                  self._head_fp8())

    def _head_fp8(self):
        """The FP8 state when the LM head runs in FP8, else None."""
        return getattr(self, "fp8_state", None) if getattr(self, "fp8_head", False) else None


def cross_entropy_loss(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """-mean(gather(log_softmax(logits, 1), targets)) over flattened rows
    (reference cross_entropy_loss, examples/gpt-1b/src/main.rs:32-41)."""
    V = logits.shape[-1]
    lp = torch.log_softmax(logits.reshape(-1, V).float(), dim=1)
    return -lp.gather(1, targets.reshape(-1, 1)).mean()
