"""Fused linear cross-entropy vs the restatement of the reference's tiled LCE
and its custom VJP (rig/kernels/linear_cross_entropy.py:115-302), including the
reference test suite's edge cases: invalid targets, semantic < storage vocab,
ragged vocabularies."""

import math

import pytest
import torch

from oracle import reference_step as ref
from rig_b200 import ops
from rig_b200.kernels import tiled_tied_cross_entropy_losses

pytestmark = pytest.mark.gpu


def _rel(x, y):
    return ((x.float() - y.float()).norm() / max(y.float().norm().item(), 1e-30)).item()


def _case(cuda, n, d, v, sv, seed=0, invalid=()):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(n, d, generator=g).bfloat16()
    e = (0.02 * torch.randn(v, d, generator=g)).bfloat16()
    t = torch.randint(0, sv, (n,), generator=g, dtype=torch.int32)
    for i in invalid:
        t[i] = -1 if i % 2 else sv + 3
    cot = torch.rand(n, generator=g)
    hh = h.float().requires_grad_(True)
    ee = e.float().requires_grad_(True)
    losses = ref.TiledLinearCrossEntropy.apply(hh, ee, t, sv, torch.bfloat16)
    finite = torch.isfinite(losses)
    (losses[finite] * cot[finite]).sum().backward()
    hd, ed, td = h.to(cuda), e.to(cuda), t.to(cuda)
    lo = torch.empty(n, device=cuda)
    lse = torch.empty(n, device=cuda)
    mean = torch.empty(1, device=cuda)
    ops.lce_fwd(hd, ed, td, sv, lo, lse, mean)
    dh = torch.empty_like(hd)
    de = torch.zeros(v, d, device=cuda)
    ops.lce_bwd(hd, ed, td, lse, cot.to(cuda), sv, dh, de)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    return (lo.cpu(), mean.cpu(), dh.cpu(), de.cpu()), (losses, hh.grad, ee.grad), t


@pytest.mark.parametrize("n,d,v,sv", [(512, 256, 1000, 1000), (300, 768, 50304, 50257),
                                      (128, 64, 264, 259), (2048, 256, 50304, 50304)])
def test_values_and_grads(cuda, n, d, v, sv):
    (lo, mean, dh, de), (l_ref, dh_ref, de_ref), _ = _case(cuda, n, d, v, sv)
    assert torch.allclose(lo, l_ref.detach(), rtol=1e-4, atol=2e-4)
    assert math.isclose(mean.item(), l_ref.mean().item(), rel_tol=1e-5)
    assert _rel(dh, dh_ref) < 1e-2
    assert _rel(de, de_ref) < 1e-2
    # storage rows at or above the semantic vocabulary receive exactly zero
    assert torch.count_nonzero(de[sv:]) == 0


def test_invalid_targets(cuda):
    (lo, mean, dh, de), (l_ref, dh_ref, de_ref), t = _case(cuda, 256, 128, 1000, 900,
                                                          invalid=(3, 10, 11, 200))
    bad = (t < 0) | (t >= 900)
    assert torch.isinf(lo[bad]).all() and (lo[bad] > 0).all()
    assert torch.isfinite(lo[~bad]).all()
    assert math.isinf(mean.item())
    assert torch.count_nonzero(dh[bad]) == 0
    assert torch.allclose(lo[~bad], l_ref[~bad].detach(), rtol=1e-4, atol=2e-4)
    assert _rel(dh, dh_ref) < 1e-2
    assert _rel(de, de_ref) < 1e-2


def test_plugin_api_matches_and_validates(cuda):
    h = torch.randn(2, 64, 128, device=cuda).bfloat16().requires_grad_(True)
    e = (0.02 * torch.randn(520, 128, device=cuda)).requires_grad_(True)
    t = torch.randint(0, 500, (2, 64), device=cuda)
    losses = tiled_tied_cross_entropy_losses(h, e, t, semantic_vocab_size=500)
    assert losses.shape == (2, 64) and losses.dtype == torch.float32
    losses.mean().backward()
    assert h.grad.dtype == torch.bfloat16 and e.grad.dtype == torch.float32
    with pytest.raises(ValueError):
        tiled_tied_cross_entropy_losses(h, e, t[:, :3], semantic_vocab_size=500)
    with pytest.raises(ValueError):
        tiled_tied_cross_entropy_losses(h, e, t, semantic_vocab_size=521)
    with pytest.raises(TypeError):
        tiled_tied_cross_entropy_losses(h, e, t.float(), semantic_vocab_size=500)
    with pytest.raises(ValueError):
        tiled_tied_cross_entropy_losses(h, e, t, semantic_vocab_size=500, vocab_tile_size=0)
