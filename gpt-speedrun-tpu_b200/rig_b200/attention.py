"""Attention runtime helpers with the reference's names (rig/attention.py)."""

from __future__ import annotations

from .kernels.flash_attention import AttentionConfig, make_causal_attention
from . import ops


def attention_softmax_scale(rule: str, head_dim: int) -> float:
    """rig/attention.py:55-62."""

    if rule == "inverse_head_dim":
        return 1.0 / float(head_dim)
    if rule == "inverse_sqrt_head_dim":
        return head_dim ** -0.5
    raise ValueError(f"unsupported attention scale {rule!r}")


def make_mesh_attention(*, backend: str = "b200_flash", softmax_scale: float, mesh=None,
                        tiles=None, document_masking: bool = False):
    """rig/attention.py:165-202. With one process per GPU the batch is already
    rank-local, so no shard_map wrapper is needed: the kernel callable is
    returned directly. `None` for the dense backend, like the reference. With
    document masking the callable takes the segment ids as a fourth argument."""

    if backend == "dense":
        return None
    del document_masking  # the same callable serves both; segment ids are explicit
    return make_causal_attention(AttentionConfig(backend="b200_flash", softmax_scale=softmax_scale))


def document_segments(tokens, boundary_token: int):
    """rig/attention.py:205-208: each token's document index within its window
    (int32 [batch, seq] on the tokens' device)."""

    import torch

    return ops.document_segments(torch.as_tensor(tokens).to(torch.int32), boundary_token)
