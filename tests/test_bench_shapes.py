"""Parity at the shapes the benchmark runs, against the CPU restatement of the
reference (oracle/reference_step.py):

* the whole 125M-tier step (12 layers, d 768, 12 heads, tied vocabulary 50304,
  T 1024) at local batch 8: forward loss within 1e-3 relative, every
  per-tensor gradient within 2e-2 relative L2 (recipes/reference/train.py:
  1096-1216, 1362-1457). 8192 tokens per step make the weight gradients split
  K over CTAs, so the ordered split-K reduction is on this path;
* the fused linear cross-entropy at the reference kernel benchmark's shape
  (8192 tokens, d 768, storage vocabulary 50304, semantic 50257;
  rig/kernels/linear_cross_entropy.py:115-302), and at 40,000 tokens so that
  the backward runs its 16,384-row chunk loop three times;
* causal flash attention at BASELINE config 3 (batch 16, 12 heads, T 1024,
  head_dim 64, RoPE on q/k; rig/kernels/tpu_flash_attention.py:171-207).
"""

import math

import numpy as np
import pytest
import torch

from oracle import reference_step as ref
from rig_b200 import ops
from rig_b200.config import load_config
from rig_b200.model import GPTTrainer, init_params
from rig_b200.tokens import zipf_tokens

pytestmark = pytest.mark.gpu


def _rel(x, y):
    x, y = torch.as_tensor(x).double(), torch.as_tensor(y).double()
    return ((x - y).norm() / max(y.norm().item(), 1e-30)).item()


def test_125m_step_loss_and_grads(cuda):
    torch.set_num_threads(max(1, torch.get_num_threads()))
    cfg = load_config("baseline_125m")
    b = 8
    params = init_params(cfg, 3)
    toks = zipf_tokens(b * (cfg.seq_len + 1), cfg.vocab_size, 3).astype(np.int32)
    w = toks.reshape(b, cfg.seq_len + 1)
    x, y = np.ascontiguousarray(w[:, :-1]), np.ascontiguousarray(w[:, 1:])
    tr = GPTTrainer(cfg, b, cuda)
    tr.load_params(params)
    tr.set_batch(torch.from_numpy(x).to(cuda), torch.from_numpy(y).to(cuda))
    tr.forward()
    tr.backward()
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    loss = tr.loss.item()
    grads = tr.export(tr.grads)
    del tr
    torch.cuda.empty_cache()
    loss_ref, grads_ref = ref.loss_and_grads(params, x, y, cfg)
    assert abs(loss - loss_ref) / abs(loss_ref) < 1e-3, (loss, loss_ref)
    worst = {k: _rel(grads[k], g) for k, g in grads_ref.items()}
    bad = {k: v for k, v in worst.items() if v > 2e-2}
    assert not bad, sorted(bad.items(), key=lambda kv: -kv[1])[:5]


def _lce(cuda, n, d, v, sv, seed):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(n, d, generator=g).bfloat16()
    e = (0.02 * torch.randn(v, d, generator=g)).bfloat16()
    t = torch.from_numpy(zipf_tokens(n, sv, seed).astype(np.int32))
    cot = torch.full((n,), 1.0 / n)
    hh = h.float().requires_grad_(True)
    ee = e.float().requires_grad_(True)
    losses = ref.TiledLinearCrossEntropy.apply(hh, ee, t, sv, torch.bfloat16)
    (losses * cot).sum().backward()
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
    return (lo.cpu(), mean.item(), dh.cpu(), de.cpu()), (losses.detach(), hh.grad, ee.grad)


@pytest.mark.parametrize("n,d,v,sv", [(8192, 768, 50304, 50257), (40000, 64, 1000, 997)])
def test_lce_benchmark_shapes(cuda, n, d, v, sv):
    (lo, mean, dh, de), (l_ref, dh_ref, de_ref) = _lce(cuda, n, d, v, sv, 1)
    assert torch.allclose(lo, l_ref, rtol=1e-4, atol=2e-4)
    assert math.isclose(mean, l_ref.mean().item(), rel_tol=1e-5)
    assert _rel(dh, dh_ref) < 1e-2
    assert _rel(de, de_ref) < 1e-2
    assert torch.count_nonzero(de[sv:]) == 0


def test_attention_config3(cuda):
    b, h, t, scale = 16, 12, 1024, 1 / 8
    g = torch.Generator().manual_seed(2)
    q, k, v, do = (torch.randn(b, h, t, 64, generator=g).bfloat16() for _ in range(4))
    qq, kk, vv = (x.float().requires_grad_(True) for x in (q, k, v))
    qr = ref.apply_rotary(qq.bfloat16().transpose(1, 2)).transpose(1, 2)
    kr = ref.apply_rotary(kk.bfloat16().transpose(1, 2)).transpose(1, 2)
    o_ref = ref.causal_attention(qr.bfloat16(), kr.bfloat16(), vv.bfloat16(), scale)
    (o_ref.float() * do.float()).sum().backward()
    tables = ops.rope_tables(t, 64, cuda)
    qd, kd, vd, dod = (x.to(cuda) for x in (q, k, v, do))
    ops.rope_apply(qd.transpose(1, 2), tables)
    ops.rope_apply(kd.transpose(1, 2), tables)
    o = torch.empty_like(qd)
    lse = torch.empty(b, h, t, device=cuda)
    ops.attention_fwd(qd, kd, vd, o, lse, scale=scale)
    dq, dk, dv = torch.empty_like(qd), torch.empty_like(kd), torch.empty_like(vd)
    ops.attention_bwd(qd, kd, vd, o, dod, lse, dq, dk, dv, scale=scale, rope=tables)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    for name, x, y in zip(("o", "dq", "dk", "dv"), (o, dq, dk, dv),
                          (o_ref, qq.grad, kk.grad, vv.grad)):
        assert _rel(x.cpu().float(), y.float()) < 2e-2, name
