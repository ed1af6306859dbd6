"""Fused CompleteP AdamW vs the restatement of train.py:1362-1457."""

import numpy as np
import pytest
import torch

from oracle import reference_step as ref
from rig_b200 import ops
from rig_b200.config import load_config
from rig_b200.model import GPTTrainer, init_params

pytestmark = pytest.mark.gpu


def test_three_updates_match(cuda):
    cfg = load_config("smoke_parity").replace(grad_clip=0.5)
    params = init_params(cfg, 1)
    tr = GPTTrainer(cfg, 1, cuda)
    tr.load_params(params)
    rng = np.random.default_rng(0)
    p, m, v = dict(params), {k: np.zeros_like(a) for k, a in params.items()}, None
    v = {k: np.zeros_like(a) for k, a in params.items()}
    for step in range(1, 4):
        grads = {k: (rng.standard_normal(a.shape) * 1e-3).astype(np.float32) for k, a in params.items()}
        for s in tr.layout.slots:
            tr.grads[s.offset:s.offset + s.size].copy_(torch.from_numpy(grads[s.name].reshape(-1)))
        tr.loss.fill_(float(step))
        tr.optimizer_step()
        p, m, v, lr, gn = ref.adamw_update(p, m, v, grads, step, cfg)
        torch.cuda.synchronize()
        row = tr.history[step - 1].cpu().numpy()
        assert row[0] == step
        np.testing.assert_allclose(row[1], lr, rtol=1e-6)
        np.testing.assert_allclose(row[2], gn, rtol=1e-5)
    got = tr.export()
    for k in params:
        np.testing.assert_allclose(got[k], p[k], rtol=2e-5, atol=1e-7, err_msg=k)
    bf = tr.export(tr.params_bf16)
    for k in params:
        assert np.array_equal(bf[k], torch.from_numpy(got[k]).bfloat16().float().numpy()), k
