"""Attention runtime helpers with the reference's names (rig/attention.py)."""

from __future__ import annotations

from .kernels.flash_attention import AttentionConfig, make_causal_attention


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
    returned directly. `None` for the dense backend, like the reference."""

    if backend == "dense":
        return None
    if document_masking:
        raise NotImplementedError("document masking is not supported yet")
    return make_causal_attention(AttentionConfig(backend="b200_flash", softmax_scale=softmax_scale))
