"""Model families: the GPT decoder of the reference example (CPU reference path
and fused sm_100a path) and synthetic data."""
from .data import SyntheticDataLoader  # noqa: F401
from .gpt import (FeedForward, GptConfig, GptModel, MultiHeadAttention, TransformerBlock,  # noqa: F401
                  create_causal_mask, create_position_ids, cross_entropy_loss)
