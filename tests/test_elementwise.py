"""Memory-bound kernels vs fp32 PyTorch restatements of rig/nn.py and train.py."""

import numpy as np
import pytest
import torch

from oracle import reference_step as ref
from rig_b200 import ops

pytestmark = pytest.mark.gpu


def _rel(x, y):
    return ((x.float() - y.float()).norm() / y.float().norm()).item()


@pytest.mark.parametrize("rows,d", [(1000, 768), (37, 256), (8, 2048), (5, 3072)])
def test_rms_norm_fwd(cuda, rows, d):
    x = torch.randn(rows, d).bfloat16()
    s = (1 + 0.1 * torch.randn(d)).bfloat16()
    y = torch.empty(rows, d, device=cuda, dtype=torch.bfloat16)
    r = torch.empty(rows, device=cuda)
    ops.rms_norm_fwd(x.to(cuda), s.to(cuda), y, r)
    expect = ref.rms_norm(x, s)
    assert _rel(y.cpu(), expect) < 5e-3
    x32 = x.float()
    assert torch.allclose(r.cpu(), torch.rsqrt((x32 * x32).mean(-1) + 1e-5), rtol=1e-5)


@pytest.mark.parametrize("rows,d", [(1000, 768), (64, 256), (8, 2048)])
def test_rms_norm_bwd(cuda, rows, d):
    x = torch.randn(rows, d).bfloat16()
    s = (1 + 0.1 * torch.randn(d)).bfloat16()
    dy = torch.randn(rows, d).bfloat16()
    dres = torch.randn(rows, d).bfloat16()
    # autograd of the restatement, fp32 end to end
    xx = x.float().requires_grad_(True)
    ss = s.float().requires_grad_(True)
    y = xx * torch.rsqrt((xx * xx).mean(-1, keepdim=True) + 1e-5) * ss
    (y * dy.float()).sum().backward()
    xd, sd, dyd = x.to(cuda), s.to(cuda), dy.to(cuda)
    yy = torch.empty_like(xd)
    r = torch.empty(rows, device=cuda)
    ops.rms_norm_fwd(xd, sd, yy, r)
    dx = dres.to(cuda).clone()
    dscale = torch.zeros(d, device=cuda)
    colsum = torch.full((d,), 0.5, device=cuda)
    ops.rms_norm_bwd(xd, sd, r, dyd, dx, dx, dscale, colsum, 0.25)
    assert _rel(dx.cpu().float() - dres.float(), xx.grad) < 1e-2
    assert _rel(dscale.cpu(), ss.grad) < 1e-2
    # fused bias gradient: += alpha * column sums of the stored bf16 dx_out
    expect = 0.5 + 0.25 * dx.cpu().float().sum(0)
    assert torch.allclose(colsum.cpu(), expect, rtol=1e-4, atol=1e-3)


def test_embedding(cuda):
    v, d, n = 1000, 256, 4096
    table = torch.randn(v, d).bfloat16()
    tok = torch.randint(0, v, (n,), dtype=torch.int32)
    out = torch.empty(n, d, device=cuda, dtype=torch.bfloat16)
    ops.embedding_fwd(tok.to(cuda), table.to(cuda), out)
    assert torch.equal(out.cpu(), table[tok.long()])
    dout = torch.randn(n, d).bfloat16()
    dt = torch.zeros(v, d, device=cuda)
    ops.embedding_bwd(tok.to(cuda), dout.to(cuda), dt)
    expect = torch.zeros(v, d).index_add_(0, tok.long(), dout.float())
    assert torch.allclose(dt.cpu(), expect, atol=1e-4)


def _skewed_tokens(n, vocab, seed):
    """Zipf-like ids (a few tokens own long runs that cross many blocks of the
    sorted order), plus a block of one repeated id and a few invalid ids."""

    g = torch.Generator().manual_seed(seed)
    ranks = torch.multinomial(1.0 / torch.arange(1, vocab + 1).float() ** 1.1, n, replacement=True,
                              generator=g)
    tok = ranks.to(torch.int32)
    tok[n // 3 : n // 3 + 3000] = 7  # one id in 3000 consecutive rows
    tok[5] = -1
    tok[n - 2] = vocab  # outside [0, vocab): contributes nothing
    return tok


@pytest.mark.parametrize("n,d,vocab", [(131072, 768, 50304), (5000, 8, 70000), (333, 64, 256),
                                       (1, 16, 10)])
def test_embedding_bwd_ordered(cuda, n, d, vocab):
    """The sorted scatter matches an fp64 index_add (invalid ids dropped), adds
    into the existing table, and repeats bit for bit."""

    tok = _skewed_tokens(n, vocab, 3) if n > 1 else torch.tensor([4], dtype=torch.int32)
    dout = torch.randn(n, d, generator=torch.Generator().manual_seed(4)).bfloat16()
    base = torch.randn(vocab, d, generator=torch.Generator().manual_seed(5))
    outs = []
    for _ in range(2):
        dt = base.to(cuda)
        ops.embedding_bwd(tok.to(cuda), dout.to(cuda), dt)
        outs.append(dt.cpu())
    torch.cuda.synchronize()
    valid = (tok >= 0) & (tok < vocab)
    expect = base.double().index_add_(0, tok[valid].long(), dout[valid].double())
    assert torch.allclose(outs[0].double(), expect, atol=2e-3 + 1e-5 * expect.abs().max().item())
    assert torch.equal(outs[0], outs[1])


def test_rope_tables(cuda):
    cos, sin = ops.rope_tables(1024, 64, cuda)
    ec, es = ref.rope_tables(1024, 64)
    # cos/sin are rounded to bf16 exactly like the restatement (one-ulp ties allowed)
    assert (cos.cpu().float() - ec.float()).abs().max().item() <= 2 ** -8
    assert (sin.cpu().float() - es.float()).abs().max().item() <= 2 ** -8
    assert (cos.cpu() != ec).float().mean().item() < 1e-3


@pytest.mark.parametrize("rows,n", [(131, 768), (4096, 2304), (10, 8)])
def test_colsum(cuda, rows, n):
    x = torch.randn(rows, n).bfloat16()
    out = torch.full((n,), 1.0, device=cuda)
    ops.colsum(x.to(cuda), out, alpha=0.5)
    assert torch.allclose(out.cpu(), 1.0 + 0.5 * x.float().sum(0), atol=1e-3, rtol=1e-4)


def test_reductions_repeat_bit_for_bit(cuda):
    """RMSNorm-backward column reductions and colsum add per-block partials in
    a fixed order: two calls on the same inputs agree exactly."""

    rows, d = 131072, 768
    g = torch.Generator().manual_seed(9)
    x = torch.randn(rows, d, generator=g).bfloat16().to(cuda)
    s = (1 + 0.1 * torch.randn(d, generator=g)).bfloat16().to(cuda)
    dy = torch.randn(rows, d, generator=g).bfloat16().to(cuda)
    y = torch.empty_like(x)
    r = torch.empty(rows, device=cuda)
    ops.rms_norm_fwd(x, s, y, r)
    res = []
    for _ in range(2):
        dx = torch.empty_like(x)
        dscale = torch.zeros(d, device=cuda)
        col = torch.zeros(d, device=cuda)
        ops.rms_norm_bwd(x, s, r, dy, None, dx, dscale, col, 0.5)
        cs = torch.zeros(3 * d, device=cuda)
        ops.colsum(torch.cat([dx, dx, dx], 1), cs, 2.0)
        res.append((dscale.cpu(), col.cpu(), cs.cpu()))
    for a, b in zip(*res):
        assert torch.equal(a, b)
    assert torch.allclose(res[0][2], 4.0 * res[0][1].repeat(3), rtol=1e-5, atol=1e-2)


@pytest.mark.parametrize("n", [1, 7, 4096, 100003])
def test_cast(cuda, n):
    x = torch.randn(n)
    y = torch.empty(n, device=cuda, dtype=torch.bfloat16)
    ops.cast_bf16(x.to(cuda), y)
    assert torch.equal(y.cpu(), x.bfloat16())


def test_apply_rotary_plugin_and_backward(cuda):
    """rig_b200.nn.apply_rotary (rig/nn.py:36-52): forward equals the
    restatement, and its gradient is the transpose rotation."""

    from rig_b200 import nn

    x = torch.randn(2, 300, 3, 64).bfloat16()
    want = ref.apply_rotary(x)
    xd = x.to(cuda).requires_grad_(True)
    y = nn.apply_rotary(xd)
    assert _rel(y.detach().cpu(), want) < 5e-3
    dy = torch.randn_like(x)
    y.backward(dy.to(cuda))
    xx = x.float().requires_grad_(True)
    ref.apply_rotary(xx).float().backward(dy.float())
    assert _rel(xd.grad.cpu(), xx.grad) < 1e-2
    with pytest.raises(ValueError):
        nn.apply_rotary(torch.zeros(2, 3, 4, device=cuda))


def test_device_error_flags(cuda):
    """A token id outside the vocabulary reaches the gather: the embedding
    family's flag is raised (and cleared by the read), nothing traps."""

    from rig_b200 import _lib

    assert _lib.load().gptb200_device_error_flags(1) == 0
    table = torch.randn(100, 64, device=cuda).bfloat16()
    tok = torch.tensor([3, 100, 5], dtype=torch.int32, device=cuda)
    out = torch.empty(3, 64, device=cuda, dtype=torch.bfloat16)
    ops.embedding_fwd(tok, table, out)
    assert _lib.load().gptb200_device_error_flags(1) == _lib.DEVERR_TOKEN_RANGE
    assert ops.device_error() == 0
