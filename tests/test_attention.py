"""Flash attention (RoPE fused on load) vs the dense restatement of
reference_causal_attention (rig/kernels/tpu_flash_attention.py:171-207)."""

import numpy as np
import pytest
import torch

from oracle import reference_step as ref
from rig_b200 import ops

pytestmark = pytest.mark.gpu


def _rel(x, y):
    return ((x.float() - y.float()).norm() / y.float().norm()).item()


def _run(cuda, b, h, t, rope, seed=0, scale=1 / 64):
    g = torch.Generator().manual_seed(seed)
    q, k, v, do = (torch.randn(b, h, t, 64, generator=g).bfloat16() for _ in range(4))
    # restatement: RoPE on BTHD, then dense causal attention in fp32 with bf16 P
    qq = q.float().requires_grad_(True)
    kk = k.float().requires_grad_(True)
    vv = v.float().requires_grad_(True)
    qr, kr = qq, kk
    if rope:
        qr = ref.apply_rotary(qq.bfloat16().transpose(1, 2)).transpose(1, 2)
        kr = ref.apply_rotary(kk.bfloat16().transpose(1, 2)).transpose(1, 2)
    o_ref = ref.causal_attention(qr.bfloat16(), kr.bfloat16(), vv.bfloat16(), scale)
    (o_ref.float() * do.float()).sum().backward()
    tables = ops.rope_tables(t, 64, cuda) if rope else None
    qd, kd, vd, dod = (x.to(cuda) for x in (q, k, v, do))
    if rope:  # q/k are rotated before the kernel; its backward rotates dq/dk back
        ops.rope_apply(qd.transpose(1, 2), tables)
        ops.rope_apply(kd.transpose(1, 2), tables)
    o = torch.empty_like(qd)
    lse = torch.empty(b, h, t, device=cuda)
    ops.attention_fwd(qd, kd, vd, o, lse, scale=scale)
    dq, dk, dv = torch.empty_like(qd), torch.empty_like(kd), torch.empty_like(vd)
    ops.attention_bwd(qd, kd, vd, o, dod, lse, dq, dk, dv, scale=scale, rope=tables)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    return (o.cpu(), dq.cpu(), dk.cpu(), dv.cpu()), (o_ref, qq.grad, kk.grad, vv.grad)


@pytest.mark.parametrize("rope", [False, True])
@pytest.mark.parametrize("b,h,t", [(2, 3, 256), (1, 2, 1024), (1, 1, 200), (2, 1, 64),
                                   (1, 1, 128), (1, 2, 384), (1, 1, 1000)])
def test_fwd_bwd_vs_restatement(cuda, b, h, t, rope):
    got, want = _run(cuda, b, h, t, rope)
    names = ("o", "dq", "dk", "dv")
    for name, x, y in zip(names, got, want):
        assert _rel(x, y) < 2e-2, name


def test_sqrt_scale(cuda):
    got, want = _run(cuda, 1, 2, 384, False, seed=3, scale=64 ** -0.5)
    for x, y in zip(got, want):
        assert _rel(x, y) < 2e-2


def test_bthd_strided_layout(cuda):
    """Packed [B, T, 3, H, 64] qkv buffer (the step's layout) gives the same result."""

    b, h, t = 2, 4, 256
    qkv = torch.randn(b, t, 3, h, 64, device=cuda).bfloat16()
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    o = torch.empty(b, t, h, 64, device=cuda, dtype=torch.bfloat16)
    lse = torch.empty(b, h, t, device=cuda)
    ops.attention_fwd(q, k, v, o, lse, scale=1 / 64, layout="bthd")
    qc, kc, vc = (x.transpose(1, 2).contiguous() for x in (q, k, v))
    o2 = torch.empty_like(qc)
    lse2 = torch.empty_like(lse)
    ops.attention_fwd(qc, kc, vc, o2, lse2, scale=1 / 64)
    assert torch.equal(o.transpose(1, 2), o2)
    assert torch.equal(lse, lse2)


def test_rope_apply_matches_restatement(cuda):
    x = torch.randn(2, 300, 3, 64).bfloat16()
    tables = ops.rope_tables(300, 64, cuda)
    xd = x.to(cuda)
    ops.rope_apply(xd, tables)
    want = ref.apply_rotary(x)
    assert (xd.cpu().float() - want.float()).abs().max().item() <= 2 ** -7 * want.abs().max().item()
    ops.rope_apply(xd, tables, inverse=True)  # the transpose rotation undoes it (to rounding)
    assert _rel(xd.cpu(), x) < 1e-2


def test_qkv_rope_epilogue(cuda):
    """The QKV GEMM epilogue applies bias + RoPE to the q/k columns only."""

    from rig_b200 import _lib
    n_tok, t, d = 512, 256, 128
    x = torch.randn(n_tok, d, device=cuda).bfloat16()
    w = (0.1 * torch.randn(d, 3 * d, device=cuda)).bfloat16()
    bias = (0.1 * torch.randn(3 * d, device=cuda)).bfloat16()
    tables = ops.rope_tables(t, 64, cuda)
    out = torch.empty(n_tok, 3 * d, device=cuda, dtype=torch.bfloat16)
    ops.matmul(x, w, bias=bias, out=out, kind=_lib.EPI_BIAS_ROPE, rope=tables, rope_cols=2 * d)
    plain = ops.matmul(x, w, bias=bias)
    pl = plain.view(n_tok // t, t, 3, d // 64, 64).clone()
    ops.rope_apply(pl[:, :, 0], tables)
    ops.rope_apply(pl[:, :, 1], tables)
    o = out.view_as(pl).float()
    assert ((o - pl.float()).abs() <= 2 ** -7 * pl.float().abs() + 1e-6).all()


def _segments(b, t, kind, seed):
    rng = np.random.default_rng(seed)
    if kind == "one":
        return np.zeros((b, t), np.int32)
    if kind == "random":  # arbitrary ids: the semantics are plain id equality
        return rng.integers(0, 3, (b, t)).astype(np.int32)
    p = {"docs300": 1 / 300, "docs40": 1 / 40}[kind]
    return ref.document_segments(rng.random((b, t)) < p, True)


@pytest.mark.parametrize("kind", ["one", "docs300", "docs40", "random"])
@pytest.mark.parametrize("b,h,t", [(2, 2, 1024), (1, 2, 1000), (1, 1, 200), (2, 1, 2048)])
def test_document_masking_vs_restatement(cuda, kind, b, h, t):
    """Segment ids (rig/attention.py:205-208; reference_causal_attention's
    segment_ids): forward and all three gradients, with and without block
    skipping, including ids that are not monotone."""

    g = torch.Generator().manual_seed(11)
    q, k, v, do = (torch.randn(b, h, t, 64, generator=g).bfloat16() for _ in range(4))
    seg = _segments(b, t, kind, 5)
    qq, kk, vv = (x.float().requires_grad_(True) for x in (q, k, v))
    o_ref = ref.causal_attention(qq.bfloat16(), kk.bfloat16(), vv.bfloat16(), 1 / 64, seg)
    (o_ref.float() * do.float()).sum().backward()
    qd, kd, vd, dod = (x.to(cuda) for x in (q, k, v, do))
    segd = torch.from_numpy(seg).to(cuda)
    o = torch.empty_like(qd)
    lse = torch.empty(b, h, t, device=cuda)
    ops.attention_fwd(qd, kd, vd, o, lse, scale=1 / 64, segment_ids=segd)
    dq, dk, dv = torch.empty_like(qd), torch.empty_like(kd), torch.empty_like(vd)
    ops.attention_bwd(qd, kd, vd, o, dod, lse, dq, dk, dv, scale=1 / 64, segment_ids=segd)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    for name, x, y in zip(("o", "dq", "dk", "dv"), (o, dq, dk, dv),
                          (o_ref, qq.grad, kk.grad, vv.grad)):
        assert _rel(x.cpu(), y) < 2e-2, (name, _rel(x.cpu(), y))


def test_single_segment_equals_causal(cuda):
    g = torch.Generator().manual_seed(2)
    q, k, v = (torch.randn(1, 2, 512, 64, generator=g).bfloat16().to(cuda) for _ in range(3))
    outs = []
    for seg in (None, torch.full((1, 512), 7, dtype=torch.int32, device=cuda)):
        o = torch.empty_like(q)
        lse = torch.empty(1, 2, 512, device=cuda)
        ops.attention_fwd(q, k, v, o, lse, scale=1 / 64, segment_ids=seg)
        outs.append((o.cpu(), lse.cpu()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
