"""Tensor-level wrappers over the libgptb200 C ABI.

Each function takes CUDA torch tensors (PyTorch is used for device memory and
streams only), checks dtypes/shapes/contiguity on the host, and launches the
kernel on the current torch stream. No function here has a CPU path: a CPU
tensor raises ``ValueError``.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import Epilogue, call

BF16 = torch.bfloat16
F32 = torch.float32


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("rig_b200 kernels need CUDA tensors (there is no CPU path)")


def _row_major(t: torch.Tensor, name: str) -> int:
    """Returns the leading dimension of a 2-D tensor with unit inner stride."""

    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D tensor with contiguous rows, got {tuple(t.stride())}")
    return t.stride(0)


# ----------------------------------------------------------------- GEMM
def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    out: torch.Tensor,
    *,
    a_mn_major: bool = False,
    b_mn_major: bool = False,
    m: int,
    n: int,
    k: int,
    kind: int = _lib.EPI_BF16,
    alpha: float = 1.0,
    bias: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    aux: torch.Tensor | None = None,
    accumulate: bool = False,
    rope: tuple[torch.Tensor, torch.Tensor] | None = None,
    rope_cols: int = 0,
    row_range: torch.Tensor | None = None,
    range_dim: int = 0,
    workspace: torch.Tensor | None = None,
) -> torch.Tensor:
    """out[m, n] = epilogue(sum_k A[m, k] B[n, k]); see include/gptb200.h.
    row_range: optional int32 device tensor {offset, count} restricting the M
    rows (range_dim 1) or the K rows (range_dim 2) that take part.
    workspace: scratch of EPI_F32_SPLITK (allocated here when not given)."""

    _cuda(a, b, out, bias, residual, aux, row_range, workspace)
    if kind == _lib.EPI_F32_SPLITK and workspace is None:
        workspace = splitk_workspace(gemm_workspace_size(m, n, k, kind), out.device)
    if a.dtype != BF16 or b.dtype != BF16:
        raise TypeError("GEMM operands must be bfloat16")
    lda, ldb, ldc = _row_major(a, "a"), _row_major(b, "b"), _row_major(out, "out")
    epi = Epilogue(
        kind=kind,
        accumulate=int(accumulate),
        alpha=float(alpha),
        bias=_ptr(bias),
        residual=_ptr(residual),
        ld_residual=0 if residual is None else _row_major(residual, "residual"),
        aux=_ptr(aux),
        ld_aux=0 if aux is None else _row_major(aux, "aux"),
        rope_cos=None if rope is None else rope[0].data_ptr(),
        rope_sin=None if rope is None else rope[1].data_ptr(),
        rope_seq=0 if rope is None else rope[0].shape[0],
        rope_cols=int(rope_cols),
        row_range=_ptr(row_range),
        range_dim=int(range_dim) if row_range is not None else 0,
        workspace=_ptr(workspace),
    )
    if gemm_timer is not None:
        start = torch.cuda.Event(enable_timing=True)
        start.record()
    call(
        "gptb200_gemm",
        a.data_ptr(), int(a_mn_major), lda, b.data_ptr(), int(b_mn_major), ldb,
        out.data_ptr(), ldc, m, n, k, ctypes.byref(epi), _stream(),
    )
    if gemm_timer is not None and row_range is None:  # a range GEMM's work is device-side
        end = torch.cuda.Event(enable_timing=True)
        end.record()
        gemm_timer.append((start, end, 2.0 * m * n * k,
                           _gemm_algorithmic_bytes(m, n, k, kind, accumulate, bias, residual, aux)))
    return out


def _gemm_algorithmic_bytes(m, n, k, kind, accumulate, bias, residual, aux) -> int:
    """Bytes a GEMM launch must move at least: each operand read once, the
    output written once (fp32 outputs that accumulate are read as well), plus
    the epilogue's own inputs and outputs (bias, residual, GELU derivative)."""

    nbytes = 2 * (m * k + n * k)
    if kind in (_lib.EPI_F32, _lib.EPI_F32_ATOMIC, _lib.EPI_F32_SPLITK):
        reads_c = kind != _lib.EPI_F32 or bool(accumulate)
        nbytes += 4 * m * n * (2 if reads_c else 1)
    else:
        nbytes += 2 * m * n
    if kind in (_lib.EPI_BIAS_GELU, _lib.EPI_DGELU):  # gelu' written / read
        nbytes += 2 * m * n
    if residual is not None:
        nbytes += 2 * m * n
    if bias is not None:
        nbytes += 2 * n
    return nbytes


def gemm_workspace_size(m: int, n: int, k: int, kind: int) -> int:
    return int(_lib.load().gptb200_gemm_workspace_size(m, n, k, kind))


def splitk_workspace(nbytes: int, device) -> torch.Tensor | None:
    """Workspace of EPI_F32_SPLITK (the per-split partial slabs)."""

    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device) if nbytes else None


def _scratch(nbytes: int, device) -> torch.Tensor | None:
    """A fresh uint8 workspace (None when no scratch is needed)."""

    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device) if nbytes else None


# When set to a list, every gemm() call appends (start_event, end_event, flops,
# algorithmic bytes) recorded on the launching stream; the benchmark uses it to time the GEMM
# launches inside its measured steps.
gemm_timer: list | None = None


def launch_count() -> int:
    """Kernels launched by libgptb200 in this process so far."""

    return int(_lib.load().gptb200_launch_count())


def matmul(x: torch.Tensor, w: torch.Tensor, *, bias=None, out=None, kind=_lib.EPI_BF16,
           alpha=1.0, residual=None, aux=None, rope=None, rope_cols=0) -> torch.Tensor:
    """y[M, N] = x[M, K] @ w[K, N] (w in the reference's [in, out] layout)."""

    m, k = x.shape
    n = w.shape[1]
    if out is None:
        out = torch.empty(m, n, device=x.device, dtype=BF16)
    return gemm(x, w, out, b_mn_major=True, m=m, n=n, k=k, kind=kind, alpha=alpha, bias=bias,
                residual=residual, aux=aux, rope=rope, rope_cols=rope_cols)


def rope_apply(x: torch.Tensor, rope, *, inverse: bool = False) -> torch.Tensor:
    """In-place interleaved RoPE on a BTHD view (inverse: the transpose rotation)."""

    _cuda(x)
    if x.dim() != 4 or x.stride(3) != 1:
        raise ValueError("rope_apply expects a [B, T, H, D] view with a contiguous head dim")
    b, t, h, d = x.shape
    call("gptb200_rope_apply", x.data_ptr(), x.stride(0), x.stride(1), x.stride(2), b, t, h, d,
         rope[0].data_ptr(), rope[1].data_ptr(), int(inverse), _stream())
    return x


# ----------------------------------------------------------------- RMSNorm
def rms_norm_fwd(x: torch.Tensor, scale: torch.Tensor, y: torch.Tensor, rstd: torch.Tensor):
    _cuda(x, scale, y, rstd)
    rows, d = x.shape
    call("gptb200_rms_norm_fwd", x.data_ptr(), scale.data_ptr(), y.data_ptr(), rstd.data_ptr(),
         rows, d, _stream())
    return y, rstd


def rms_norm_bwd_workspace_size(rows: int, d: int) -> int:
    return int(_lib.load().gptb200_rms_norm_bwd_workspace_size(rows, d))


def rms_norm_bwd(x, scale, rstd, dy, dx_in, dx_out, dscale, dx_colsum=None, colsum_alpha=1.0,
                 workspace=None):
    """dx_out = dx_in + d(rms_norm)/dx . dy; dscale +=; dx_colsum += alpha * colsum(dx_out)."""

    _cuda(x, scale, rstd, dy, dx_in, dx_out, dscale, dx_colsum, workspace)
    rows, d = x.shape
    if workspace is None:
        workspace = _scratch(rms_norm_bwd_workspace_size(rows, d), x.device)
    call("gptb200_rms_norm_bwd", x.data_ptr(), scale.data_ptr(), rstd.data_ptr(), dy.data_ptr(),
         _ptr(dx_in), dx_out.data_ptr(), dscale.data_ptr(), _ptr(dx_colsum),
         float(colsum_alpha), rows, d, workspace.data_ptr(), _stream())
    return dx_out


# ----------------------------------------------------------------- embedding
def embedding_fwd(tokens: torch.Tensor, table: torch.Tensor, out: torch.Tensor):
    _cuda(tokens, table, out)
    if tokens.dtype != torch.int32:
        raise TypeError("token ids must be int32")
    call("gptb200_embedding_fwd", tokens.data_ptr(), table.data_ptr(), out.data_ptr(),
         tokens.numel(), table.shape[1], table.shape[0], _stream())
    return out


def embedding_bwd_workspace_size(n: int, d: int, vocab: int) -> int:
    return int(_lib.load().gptb200_embedding_bwd_workspace_size(n, d, vocab))


def embedding_bwd(tokens: torch.Tensor, dout: torch.Tensor, dtable: torch.Tensor, workspace=None):
    """dtable[tokens[i]] += dout[i] in a fixed (token, row) order (bit-reproducible)."""

    _cuda(tokens, dout, dtable, workspace)
    if tokens.dtype != torch.int32:
        raise TypeError("token ids must be int32")
    n, (v, d) = tokens.numel(), dtable.shape
    if workspace is None:
        workspace = _scratch(embedding_bwd_workspace_size(n, d, v), dtable.device)
    call("gptb200_embedding_bwd", tokens.data_ptr(), dout.data_ptr(), dtable.data_ptr(),
         n, d, v, workspace.data_ptr(), _stream())
    return dtable


def rope_tables(seq: int, head_dim: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    cos = torch.empty(seq, head_dim // 2, device=device, dtype=BF16)
    sin = torch.empty_like(cos)
    call("gptb200_rope_tables", cos.data_ptr(), sin.data_ptr(), seq, head_dim, _stream())
    return cos, sin


def document_segments(tokens: torch.Tensor, boundary_token: int,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """rig/attention.py:205-208 on the device: cumulative boundary count per row."""

    _cuda(tokens, out)
    if tokens.dtype != torch.int32 or tokens.dim() != 2:
        raise TypeError("tokens must be an int32 [batch, seq] tensor")
    tokens = tokens.contiguous()
    if out is None:
        out = torch.empty_like(tokens)
    call("gptb200_document_segments", tokens.data_ptr(), tokens.shape[0], tokens.shape[1],
         int(boundary_token), out.data_ptr(), _stream())
    return out


# ----------------------------------------------------------------- attention
def _strides4(t: torch.Tensor, layout: str) -> tuple[int, int, int]:
    """Element strides (batch, head, time) of a rank-4 view, inner dim contiguous."""

    if t.stride(3) != 1:
        raise ValueError("attention tensors need a contiguous head dimension")
    if layout == "bhsd":
        return t.stride(0), t.stride(1), t.stride(2)
    return t.stride(0), t.stride(2), t.stride(1)  # bthd


def _segments(segment_ids, b: int, t: int):
    if segment_ids is None:
        return None
    _cuda(segment_ids)
    if segment_ids.dtype != torch.int32 or tuple(segment_ids.shape) != (b, t):
        raise ValueError(f"segment_ids must be int32 [{b}, {t}], got {segment_ids.dtype} "
                         f"{tuple(segment_ids.shape)}")
    return segment_ids.contiguous()


def attention_fwd(q, k, v, o, lse, *, scale: float, layout: str = "bhsd", segment_ids=None):
    """Causal attention; q/k/v/o are rank-4 views in `layout` ('bhsd' or 'bthd').
    q and k are used as given (apply RoPE before, e.g. with `rope_apply`).
    segment_ids: optional int32 [B, T] document ids (same-document attention)."""

    _cuda(q, k, v, o, lse)
    sb, sh, st = _strides4(q, layout)
    if _strides4(k, layout) != (sb, sh, st) or _strides4(v, layout) != (sb, sh, st):
        raise ValueError("q, k and v must share strides")
    osb, osh, ost = _strides4(o, layout)
    if layout == "bhsd":
        b, h, t, dh = q.shape
    else:
        b, t, h, dh = q.shape
    seg = _segments(segment_ids, b, t)
    call("gptb200_attention_fwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), sb, sh, st,
         o.data_ptr(), osb, osh, ost, lse.data_ptr(), b, h, t, dh, float(scale), _ptr(seg),
         _stream())
    return o, lse


def attention_workspace(b: int, h: int, t: int, device) -> torch.Tensor:
    n = _lib.load().gptb200_attention_bwd_workspace_size(b, h, t)
    return torch.empty(n, dtype=torch.uint8, device=device)


def attention_bwd(q, k, v, o, do, lse, dq, dk, dv, *, scale: float, layout="bhsd", rope=None,
                  workspace=None, segment_ids=None):
    _cuda(q, k, v, o, do, lse, dq, dk, dv)
    sb, sh, st = _strides4(q, layout)
    for t_ in (k, v, dq, dk, dv):
        if _strides4(t_, layout) != (sb, sh, st):
            raise ValueError("q, k, v, dq, dk, dv must share strides")
    osb, osh, ost = _strides4(o, layout)
    if _strides4(do, layout) != (osb, osh, ost):
        raise ValueError("o and do must share strides")
    if layout == "bhsd":
        b, h, t, dh = q.shape
    else:
        b, t, h, dh = q.shape
    if workspace is None:
        workspace = attention_workspace(b, h, t, q.device)
    cos, sin = rope if rope is not None else (None, None)
    seg = _segments(segment_ids, b, t)
    call("gptb200_attention_bwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), sb, sh, st,
         o.data_ptr(), do.data_ptr(), osb, osh, ost, lse.data_ptr(), dq.data_ptr(),
         dk.data_ptr(), dv.data_ptr(), b, h, t, dh, float(scale), _ptr(cos), _ptr(sin),
         _ptr(seg), workspace.data_ptr(), _stream())
    return dq, dk, dv


# ----------------------------------------------------------------- cross entropy
def lce_fwd_workspace(n: int, v: int, device) -> torch.Tensor:
    size = _lib.load().gptb200_lce_fwd_workspace_size(n, v)
    return torch.empty(size, dtype=torch.uint8, device=device)


def lce_bwd_workspace(n: int, v: int, device) -> torch.Tensor:
    size = _lib.load().gptb200_lce_bwd_workspace_size(n, v)
    return torch.empty(size, dtype=torch.uint8, device=device)


def lce_fwd(hidden, embedding, targets, v_semantic, losses, lse, mean=None, workspace=None):
    _cuda(hidden, embedding, targets, losses, lse, mean)
    n, d = hidden.shape
    v = embedding.shape[0]
    if workspace is None:
        workspace = lce_fwd_workspace(n, v, hidden.device)
    call("gptb200_lce_fwd", hidden.data_ptr(), embedding.data_ptr(), targets.data_ptr(), n, d, v,
         v_semantic, losses.data_ptr(), lse.data_ptr(), _ptr(mean), workspace.data_ptr(),
         _stream())
    return losses


def lce_bwd(hidden, embedding, targets, lse, dlosses, v_semantic, dhidden, dembedding,
            workspace=None):
    _cuda(hidden, embedding, targets, lse, dlosses, dhidden, dembedding)
    n, d = hidden.shape
    v = embedding.shape[0]
    if workspace is None:
        workspace = lce_bwd_workspace(n, v, hidden.device)
    call("gptb200_lce_bwd", hidden.data_ptr(), embedding.data_ptr(), targets.data_ptr(),
         lse.data_ptr(), dlosses.data_ptr(), n, d, v, v_semantic, dhidden.data_ptr(),
         dembedding.data_ptr(), workspace.data_ptr(), _stream())
    return dhidden, dembedding


# ----------------------------------------------------------------- misc
def colsum_workspace_size(rows: int, n: int) -> int:
    return int(_lib.load().gptb200_colsum_workspace_size(rows, n))


def colsum(x: torch.Tensor, out: torch.Tensor, alpha: float = 1.0, workspace=None):
    """out += alpha * x.sum(0) (fp32, fixed summation order)."""

    _cuda(x, out, workspace)
    rows, n = x.shape
    if workspace is None:
        workspace = _scratch(colsum_workspace_size(rows, n), x.device)
    call("gptb200_colsum", x.data_ptr(), rows, n, float(alpha), out.data_ptr(),
         workspace.data_ptr(), _stream())
    return out


def masked_loss_sum(losses: torch.Tensor, mask: torch.Tensor, out: torch.Tensor | None = None):
    """out = [sum(losses * mask), sum(mask)] (fp32, deterministic), on the device."""

    _cuda(losses, mask, out)
    if losses.dtype != F32 or mask.dtype != F32:
        raise TypeError("masked_loss_sum takes fp32 losses and an fp32 mask")
    if losses.numel() != mask.numel():
        raise ValueError(f"losses {tuple(losses.shape)} and mask {tuple(mask.shape)} differ in size")
    if out is None:
        out = torch.empty(2, device=losses.device, dtype=F32)
    call("gptb200_masked_loss_sum", losses.data_ptr(), mask.contiguous().data_ptr(), losses.numel(),
         out.data_ptr(), _stream())
    return out


def cast_bf16(src: torch.Tensor, dst: torch.Tensor):
    _cuda(src, dst)
    call("gptb200_cast_bf16", src.data_ptr(), dst.data_ptr(), src.numel(), _stream())
    return dst


def adamw_workspace(n: int, device) -> torch.Tensor:
    size = _lib.load().gptb200_adamw_workspace_size(n)
    return torch.empty(size, dtype=torch.uint8, device=device)


def adamw_step(params, m, v, grads, groups_dev, n_groups, cfg, step, loss, history, params_bf16,
               workspace):
    _cuda(params, m, v, grads, groups_dev, step, loss, history, params_bf16, workspace)
    call("gptb200_adamw_step", params.data_ptr(), m.data_ptr(), v.data_ptr(), grads.data_ptr(),
         params.numel(), groups_dev.data_ptr(), n_groups, ctypes.byref(cfg), step.data_ptr(),
         _ptr(loss), _ptr(history), _ptr(params_bf16), workspace.data_ptr(), _stream())


def adamw_begin(cfg, step, workspace):
    _cuda(step, workspace)
    call("gptb200_adamw_begin", ctypes.byref(cfg), step.data_ptr(), workspace.data_ptr(), _stream())


def adamw_update_range(params, m, v, grads, begin, end, groups_dev, n_groups, cfg, slot,
                       params_bf16, workspace):
    _cuda(params, m, v, grads, groups_dev, params_bf16, workspace)
    call("gptb200_adamw_update_range", params.data_ptr(), m.data_ptr(), v.data_ptr(),
         grads.data_ptr(), int(begin), int(end), groups_dev.data_ptr(), n_groups,
         ctypes.byref(cfg), int(slot), _ptr(params_bf16), workspace.data_ptr(), _stream())


def adamw_end(n_slots, cfg, step, loss, history, workspace):
    _cuda(step, loss, history, workspace)
    call("gptb200_adamw_end", int(n_slots), ctypes.byref(cfg), step.data_ptr(), _ptr(loss),
         _ptr(history), workspace.data_ptr(), _stream())


def device_error(clear: bool = True) -> int:
    return _lib.load().gptb200_device_error(int(clear))


# ----------------------------------------------------------------- routed MLP (MoE)
def moe_rows(tokens: int, top_k: int, experts: int) -> int:
    """Rows of the expert-sorted buffer (assignments + per-expert padding to 128)."""

    return int(_lib.load().gptb200_moe_rows(tokens, top_k, experts))


def moe_dispatch_workspace(tokens: int, top_k: int, experts: int, device) -> torch.Tensor:
    n = _lib.load().gptb200_moe_dispatch_workspace_size(tokens, top_k, experts)
    return torch.empty(n, dtype=torch.uint8, device=device)


def moe_route(x, router_w, logits, chosen, gate, stats):
    """logits = x . router_w (fp32), top-k `chosen` experts and their `gate`s;
    accumulates the layer's routing statistics into `stats`."""

    _cuda(x, router_w, logits, chosen, gate, stats)
    n, d = x.shape
    e = router_w.shape[1]
    call("gptb200_moe_route", x.data_ptr(), router_w.data_ptr(), n, d, e, chosen.shape[1],
         logits.data_ptr(), chosen.data_ptr(), gate.data_ptr(), stats.data_ptr(), _stream())


def moe_dispatch(chosen, x, experts, seg, total, pos, src, grouped, workspace):
    _cuda(chosen, x, seg, total, pos, src, grouped, workspace)
    n, k = chosen.shape
    call("gptb200_moe_dispatch", chosen.data_ptr(), n, k, experts, x.data_ptr(), x.shape[1],
         seg.data_ptr(), total.data_ptr(), pos.data_ptr(), src.data_ptr(), grouped.data_ptr(),
         workspace.data_ptr(), _stream())


def moe_combine(out, pos, gate, residual, alpha, x_out):
    _cuda(out, pos, gate, residual, x_out)
    n, k = pos.shape
    call("gptb200_moe_combine", out.data_ptr(), pos.data_ptr(), gate.data_ptr(),
         residual.data_ptr(), float(alpha), n, residual.shape[1], k, x_out.data_ptr(), _stream())


def moe_combine_bwd(dx, alpha, out, pos, gate, src, total, d_out, d_gate):
    _cuda(dx, out, pos, gate, src, total, d_out, d_gate)
    n, k = pos.shape
    call("gptb200_moe_combine_bwd", dx.data_ptr(), float(alpha), out.data_ptr(), pos.data_ptr(),
         gate.data_ptr(), src.data_ptr(), total.data_ptr(), n, dx.shape[1], k, d_out.data_ptr(),
         d_gate.data_ptr(), _stream())


def moe_route_bwd(x, router_w, logits, chosen, gate, d_gate, bal_grad, d_grouped, pos,
                  d_router_w, d_x):
    _cuda(x, router_w, logits, chosen, gate, d_gate, bal_grad, d_grouped, pos, d_router_w, d_x)
    n, d = x.shape
    call("gptb200_moe_route_bwd", x.data_ptr(), router_w.data_ptr(), logits.data_ptr(),
         chosen.data_ptr(), gate.data_ptr(), d_gate.data_ptr(), bal_grad.data_ptr(),
         d_grouped.data_ptr(), pos.data_ptr(), n, d, router_w.shape[1], chosen.shape[1],
         d_router_w.data_ptr(), d_x.data_ptr(), _stream())


def moe_segment_colsum(buf, seg, experts, out):
    _cuda(buf, seg, out)
    call("gptb200_moe_segment_colsum", buf.data_ptr(), seg.data_ptr(), experts, buf.shape[1],
         out.data_ptr(), _stream())


def moe_finalize(stats, layers, experts, tokens, top_k, coefficient, bwd_scale, bal_grad, loss,
                 history, step):
    _cuda(stats, bal_grad, loss, history, step)
    call("gptb200_moe_finalize", stats.data_ptr(), layers, experts, tokens, top_k,
         float(coefficient), float(bwd_scale), bal_grad.data_ptr(), loss.data_ptr(),
         history.data_ptr(), history.shape[0], step.data_ptr(), _stream())
