"""Fused tied-embedding cross entropy with the reference's API.

Drop-in for rig/kernels/linear_cross_entropy.py:308-368
(`tiled_tied_cross_entropy`, `tiled_tied_cross_entropy_losses`): same
arguments, same validation errors raised before any launch (:45-76), same
semantics (invalid target -> +inf loss and no gradient; storage rows at or
above `semantic_vocab_size` get no mass and zero gradient). The forward and
backward run the libgptb200 fused kernels (logits never stored in HBM).
`vocab_tile_size` is accepted for API compatibility; the B200 kernel tiles
the vocabulary by its own 256-wide MMA tile.
"""

from __future__ import annotations

from typing import Any

import torch

from .. import ops
from ..nn import _as_bf16

DEFAULT_VOCAB_TILE_SIZE = 2_048


def _validate_inputs(hidden, embedding, targets, semantic_vocab_size, vocab_tile_size):
    if hidden.dim() < 1:
        raise ValueError("hidden must have at least one dimension")
    if embedding.dim() != 2:
        raise ValueError(
            f"embedding must have shape [storage_vocab, width], got {tuple(embedding.shape)}")
    if hidden.shape[-1] != embedding.shape[1]:
        raise ValueError(
            "hidden width must match the embedding width; "
            f"got {hidden.shape[-1]} and {embedding.shape[1]}")
    if tuple(targets.shape) != tuple(hidden.shape[:-1]):
        raise ValueError(
            "targets must match hidden's leading dimensions; "
            f"got {tuple(targets.shape)} and {tuple(hidden.shape[:-1])}")
    if targets.dtype.is_floating_point or targets.dtype == torch.bool:
        raise TypeError(f"targets must have an integer dtype, got {targets.dtype}")
    if not 0 < semantic_vocab_size <= embedding.shape[0]:
        raise ValueError(
            "semantic_vocab_size must be in [1, storage_vocab]; "
            f"got {semantic_vocab_size} for {embedding.shape[0]} rows")
    if vocab_tile_size <= 0:
        raise ValueError(f"vocab_tile_size must be positive, got {vocab_tile_size}")


class _TiledLosses(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, embedding, targets, semantic_vocab_size):
        d = hidden.shape[-1]
        h2 = hidden.reshape(-1, d).to(torch.bfloat16).contiguous()
        e16 = _as_bf16(embedding)
        t = targets.reshape(-1).to(torch.int32).contiguous()
        n = h2.shape[0]
        losses = torch.empty(n, dtype=torch.float32, device=hidden.device)
        lse = torch.empty(n, dtype=torch.float32, device=hidden.device)
        ops.lce_fwd(h2, e16, t, semantic_vocab_size, losses, lse)
        ctx.save_for_backward(h2, e16, t, lse)
        ctx.meta = (hidden.shape, hidden.dtype, embedding.dtype, semantic_vocab_size)
        return losses.reshape(targets.shape)

    @staticmethod
    def backward(ctx, cot):
        h2, e16, t, lse = ctx.saved_tensors
        shape, hdtype, edtype, sv = ctx.meta
        dh = torch.empty_like(h2)
        de = torch.zeros(e16.shape, dtype=torch.float32, device=h2.device)
        ops.lce_bwd(h2, e16, t, lse, cot.reshape(-1).float().contiguous(), sv, dh, de)
        return dh.reshape(shape).to(hdtype), de.to(edtype), None, None


def tiled_tied_cross_entropy_losses(hidden, embedding, targets, *, semantic_vocab_size: int,
                                    vocab_tile_size: int = DEFAULT_VOCAB_TILE_SIZE,
                                    compute_dtype: Any = torch.bfloat16) -> torch.Tensor:
    """One fp32 cross-entropy value per target, without full vocabulary logits."""

    semantic_vocab_size = int(semantic_vocab_size)
    vocab_tile_size = int(vocab_tile_size)
    if compute_dtype != torch.bfloat16:
        raise TypeError("the B200 kernel computes the projection in bfloat16")
    _validate_inputs(hidden, embedding, targets, semantic_vocab_size, vocab_tile_size)
    return _TiledLosses.apply(hidden, embedding, targets, semantic_vocab_size)


def tiled_tied_cross_entropy(hidden, embedding, targets, *, semantic_vocab_size: int,
                             vocab_tile_size: int = DEFAULT_VOCAB_TILE_SIZE,
                             compute_dtype: Any = torch.bfloat16) -> torch.Tensor:
    """Mean tiled tied-embedding cross entropy in fp32."""

    losses = tiled_tied_cross_entropy_losses(
        hidden, embedding, targets, semantic_vocab_size=semantic_vocab_size,
        vocab_tile_size=vocab_tile_size, compute_dtype=compute_dtype)
    return losses.float().mean()
