"""Kernel plugins with the names of the reference's rig.kernels package."""

from .flash_attention import AttentionConfig, make_causal_attention
from .linear_cross_entropy import (
    DEFAULT_VOCAB_TILE_SIZE,
    tiled_tied_cross_entropy,
    tiled_tied_cross_entropy_losses,
)

__all__ = [
    "AttentionConfig",
    "DEFAULT_VOCAB_TILE_SIZE",
    "make_causal_attention",
    "tiled_tied_cross_entropy",
    "tiled_tied_cross_entropy_losses",
]
