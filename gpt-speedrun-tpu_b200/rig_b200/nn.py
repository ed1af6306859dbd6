"""Layer building blocks with the signatures of the reference's rig/nn.py.

`rms_norm` (rig/nn.py:26-33), `apply_rotary` (:36-52) and `linear` (:55-56)
are differentiable (torch.autograd) wrappers over the libgptb200 kernels; `normal`,
`parameter_count` and `flatten_arrays` are the reference's host helpers
(:20-23, :59-77). Inputs are CUDA tensors; there is no CPU path.
"""

from __future__ import annotations

from typing import Any, Mapping

import numpy as np
import torch

from . import _lib, ops


def normal(rng: np.random.Generator, shape: tuple[int, ...], scale: float) -> np.ndarray:
    return rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)


def _as_bf16(t: torch.Tensor) -> torch.Tensor:
    if t.dtype == torch.bfloat16:
        return t.contiguous()
    out = torch.empty(t.shape, dtype=torch.bfloat16, device=t.device)
    return ops.cast_bf16(t.contiguous().float(), out)


class _RmsNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        s16 = _as_bf16(scale)
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        ops.rms_norm_fwd(x2, s16, y, rstd)
        ctx.save_for_backward(x2, s16, rstd)
        ctx.shape = shape
        ctx.scale_dtype = scale.dtype
        return y.reshape(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, s16, rstd = ctx.saved_tensors
        dy2 = dy.reshape(x2.shape).contiguous().to(torch.bfloat16)
        dx = torch.empty_like(x2)
        dscale = torch.zeros(x2.shape[1], dtype=torch.float32, device=x2.device)
        ops.rms_norm_bwd(x2, s16, rstd, dy2, None, dx, dscale)
        return dx.reshape(ctx.shape), dscale.to(ctx.scale_dtype)


def rms_norm(x: torch.Tensor, scale: torch.Tensor, dtype: Any = torch.bfloat16) -> torch.Tensor:
    """bf16(x * rsqrt(mean(x^2) + 1e-5)) * bf16(scale), fp32 statistics."""

    if dtype != torch.bfloat16:
        raise TypeError("the B200 kernels compute rms_norm in bfloat16")
    return _RmsNorm.apply(x.to(torch.bfloat16), scale)


_ROPE_TABLES: dict[tuple, tuple[torch.Tensor, torch.Tensor]] = {}


def _rope(length: int, head_dim: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    key = (length, head_dim, str(device))
    if key not in _ROPE_TABLES:
        _ROPE_TABLES[key] = ops.rope_tables(length, head_dim, device)
    return _ROPE_TABLES[key]


class _Rotary(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        y = x.contiguous().clone()
        rope = _rope(x.shape[1], x.shape[-1], x.device)
        ops.rope_apply(y, rope)
        ctx.rope = rope
        return y

    @staticmethod
    def backward(ctx, dy):
        # the rotation is orthogonal: its transpose (inverse = 1) is the backward
        dx = dy.to(torch.bfloat16).contiguous().clone()
        ops.rope_apply(dx, ctx.rope, inverse=True)
        return dx


def apply_rotary(x: torch.Tensor) -> torch.Tensor:
    """Interleaved base-10,000 rotary positions on one [B, T, H, D] tensor.

    Pairs (2i, 2i+1) of the head dimension are rotated by the angle
    t * 10000^(-2i/D) at sequence position t, with bf16 cos/sin tables, like
    rig/nn.py:36-52. Computes in bfloat16 on the GPU (rope_apply kernel)."""

    if x.dim() != 4:
        raise ValueError(f"apply_rotary expects a [batch, seq, heads, head_dim] tensor, got {tuple(x.shape)}")
    if x.shape[-1] % 2:
        raise ValueError("rotary attention requires an even head dimension")
    return _Rotary.apply(x.to(torch.bfloat16))


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        w16, b16 = _as_bf16(weight), _as_bf16(bias)
        y = ops.matmul(x2, w16, bias=b16)
        ctx.save_for_backward(x2, w16)
        ctx.shape = shape
        ctx.dtypes = (weight.dtype, bias.dtype)
        return y.reshape(*shape[:-1], w16.shape[1])

    @staticmethod
    def backward(ctx, dy):
        x2, w16 = ctx.saved_tensors
        m, k = x2.shape
        n = w16.shape[1]
        dy2 = dy.reshape(m, n).contiguous().to(torch.bfloat16)
        dx = torch.empty_like(x2)
        ops.gemm(dy2, w16, dx, m=m, n=k, k=n)
        dw = torch.zeros(k, n, dtype=torch.float32, device=x2.device)
        ops.gemm(x2, dy2, dw, a_mn_major=True, b_mn_major=True, m=k, n=n, k=m,
                 kind=_lib.EPI_F32_SPLITK)
        db = torch.zeros(n, dtype=torch.float32, device=x2.device)
        ops.colsum(dy2, db)
        return dx.reshape(ctx.shape), dw.to(ctx.dtypes[0]), db.to(ctx.dtypes[1])


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
           dtype: Any = torch.bfloat16) -> torch.Tensor:
    """einsum('...d,df->...f', x, W.astype(dtype)) + b.astype(dtype)."""

    if dtype != torch.bfloat16:
        raise TypeError("the B200 kernels compute linear in bfloat16")
    return _Linear.apply(x.to(torch.bfloat16), weight, bias)


def parameter_count(params: Mapping[str, Any]) -> int:
    total = 0
    for value in params.values():
        total += parameter_count(value) if isinstance(value, Mapping) else int(np.prod(np.shape(value)))
    return total


def flatten_arrays(tree: Any, prefix: str = "params") -> dict[str, np.ndarray]:
    flat: dict[str, np.ndarray] = {}

    def visit(value: Any, path: str) -> None:
        if isinstance(value, Mapping):
            for key in sorted(value):
                visit(value[key], f"{path}/{key}")
        elif isinstance(value, (list, tuple)):
            for index, child in enumerate(value):
                visit(child, f"{path}/{index}")
        else:
            flat[path] = np.asarray(value)

    visit(tree, prefix)
    return flat
