"""Causal flash attention behind the reference's factory API.

Drop-in for rig/kernels/tpu_flash_attention.py:75-97 (`AttentionConfig`) and
:962-1164 (`make_causal_attention`): the returned callable takes BHSD q, k, v
(bf16, head_dim 64) and returns BHSD output, differentiable through the
libgptb200 forward/backward kernels. Validation follows `_validate_qkv`
(:145-168). Tiles are chosen by the kernel; the `tiles` field is accepted and
ignored. Optional segment ids ([batch, seq] int32, e.g. from
`rig_b200.attention.document_segments`) restrict attention to each document
(reference_causal_attention's segment_ids, :171-207).
"""

from __future__ import annotations

import dataclasses
from typing import Callable

import torch

from .. import ops


@dataclasses.dataclass(frozen=True)
class AttentionConfig:
    backend: str = "auto"
    tiles: object | None = None
    softmax_scale: float | None = None
    interpret: bool = False
    debug: bool = False

    def __post_init__(self) -> None:
        if self.backend not in ("auto", "tpu_flash", "jax_flash", "reference", "b200_flash"):
            raise ValueError(f"unknown attention backend: {self.backend!r}")
        if self.softmax_scale is not None and self.softmax_scale <= 0.0:
            raise ValueError("softmax_scale must be positive")


def _validate_qkv(q, k, v) -> None:
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k, and v must use BHSD rank-4 layout; "
                         f"got {tuple(q.shape)}, {tuple(k.shape)}, and {tuple(v.shape)}")
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError("dense causal self-attention requires identical q/k/v shapes")
    if not all(q.shape):
        raise ValueError(f"q/k/v dimensions must be nonzero, got {tuple(q.shape)}")
    if q.shape[-1] != 64:
        raise ValueError(f"the B200 kernel requires head_dim 64, got {q.shape[-1]}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise TypeError(f"q, k, and v dtypes must match; got {q.dtype}, {k.dtype}, {v.dtype}")
    if q.dtype != torch.bfloat16:
        raise TypeError(f"q, k, and v must be bfloat16, got {q.dtype}")


class _Attention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, scale, rope, segment_ids):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        if rope is not None:  # rotate copies of q and k (BHSD viewed as BTHD)
            q, k = q.clone(), k.clone()
            ops.rope_apply(q.transpose(1, 2), rope)
            ops.rope_apply(k.transpose(1, 2), rope)
        b, h, t, _ = q.shape
        o = torch.empty_like(q)
        lse = torch.empty(b, h, t, dtype=torch.float32, device=q.device)
        ops.attention_fwd(q, k, v, o, lse, scale=scale, segment_ids=segment_ids)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.scale, ctx.rope, ctx.segment_ids = scale, rope, segment_ids
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        do = do.contiguous().to(torch.bfloat16)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        ops.attention_bwd(q, k, v, o, do, lse, dq, dk, dv, scale=ctx.scale, rope=ctx.rope,
                          segment_ids=ctx.segment_ids)
        return dq, dk, dv, None, None, None


def make_causal_attention(config: AttentionConfig = AttentionConfig(), *,
                          rope_tables=None) -> Callable:
    """Returns attention(q, k, v, segment_ids=None) over BHSD bf16 tensors.

    With `rope_tables=(cos, sin)` (from `ops.rope_tables`) the interleaved
    RoPE of rig/nn.py:36-52 is applied to q and k inside the kernel.
    """

    def attention(q, k, v, segment_ids=None):
        _validate_qkv(q, k, v)
        if segment_ids is not None:
            if tuple(segment_ids.shape) != (q.shape[0], q.shape[2]):
                raise ValueError(f"segment_ids must be [batch, seq] = {(q.shape[0], q.shape[2])}, "
                                 f"got {tuple(segment_ids.shape)}")
            segment_ids = segment_ids.to(device=q.device, dtype=torch.int32).contiguous()
        scale = config.softmax_scale if config.softmax_scale is not None else q.shape[-1] ** -0.5
        return _Attention.apply(q, k, v, float(scale), rope_tables, segment_ids)

    return attention
