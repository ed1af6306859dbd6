"""Flash attention (RoPE fused on load) vs the dense restatement of
reference_causal_attention (rig/kernels/tpu_flash_attention.py:171-207)."""

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
    o = torch.empty_like(qd)
    lse = torch.empty(b, h, t, device=cuda)
    ops.attention_fwd(qd, kd, vd, o, lse, scale=scale, rope=tables)
    dq, dk, dv = torch.empty_like(qd), torch.empty_like(kd), torch.empty_like(vd)
    ops.attention_bwd(qd, kd, vd, o, dod, lse, dq, dk, dv, scale=scale, rope=tables)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    return (o.cpu(), dq.cpu(), dk.cpu(), dv.cpu()), (o_ref, qq.grad, kk.grad, vv.grad)


@pytest.mark.parametrize("rope", [False, True])
@pytest.mark.parametrize("b,h,t", [(2, 3, 256), (1, 2, 1024), (1, 1, 200), (2, 1, 64)])
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
    tables = ops.rope_tables(t, 64, cuda)
    ops.attention_fwd(q, k, v, o, lse, scale=1 / 64, layout="bthd", rope=tables)
    qc, kc, vc = (x.transpose(1, 2).contiguous() for x in (q, k, v))
    o2 = torch.empty_like(qc)
    lse2 = torch.empty_like(lse)
    ops.attention_fwd(qc, kc, vc, o2, lse2, scale=1 / 64, rope=tables)
    assert torch.equal(o.transpose(1, 2), o2)
    assert torch.equal(lse, lse2)
