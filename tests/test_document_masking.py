"""Document-masked training step (the 8k context preset's policy,
recipes/reference/train.py:1127-1131) against the CPU restatement: segment ids
computed on the device from the tokens, same-document attention in the forward
and backward kernels."""

import numpy as np
import pytest
import torch

from oracle import reference_step as ref
from rig_b200 import ops
from rig_b200.config import load_config
from rig_b200.model import GPTTrainer, init_params
from rig_b200.tokens import zipf_tokens

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("b,t,boundary", [(3, 8192, 20), (4, 1000, 0), (2, 257, 5)])
def test_document_segments_kernel(cuda, b, t, boundary):
    tok = zipf_tokens(b * t, 50304, 4).astype(np.int32).reshape(b, t)
    got = ops.document_segments(torch.from_numpy(tok).to(cuda), boundary).cpu().numpy()
    np.testing.assert_array_equal(got, ref.document_segments(tok, boundary))


def test_step_with_document_masking(cuda):
    # boundary = token id 20 of the Zipf(1.1) stream: documents of a few hundred tokens
    cfg = load_config("smoke_parity").replace(document_masking=True, document_boundary_token=20)
    params = init_params(cfg, 0)
    b, t = cfg.batch_size, cfg.seq_len
    w = zipf_tokens(b * (t + 1), cfg.vocab_size, 9).astype(np.int32).reshape(b, t + 1)
    x, y = np.ascontiguousarray(w[:, :-1]), np.ascontiguousarray(w[:, 1:])
    segs = ref.document_segments(x, 20)
    assert segs.max() >= 2  # several documents per sequence
    loss_ref, grads_ref = ref.loss_and_grads(params, x, y, cfg)
    cfg_plain = cfg.replace(document_masking=False)
    loss_plain, _ = ref.loss_and_grads(params, x, y, cfg_plain)
    assert abs(loss_plain - loss_ref) > 1e-4  # the masking changes the loss
    tr = GPTTrainer(cfg, b, cuda)
    tr.load_params(params)
    tr.set_batch(torch.from_numpy(x).to(cuda), torch.from_numpy(y).to(cuda))
    tr.forward()
    tr.backward()
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    np.testing.assert_array_equal(tr.segments.cpu().numpy(), segs)
    loss = tr.loss.item()
    assert abs(loss - loss_ref) / abs(loss_ref) < 1e-3, (loss, loss_ref)
    grads = tr.export(tr.grads)
    worst = {}
    for k, g_ref in grads_ref.items():
        denom = np.linalg.norm(g_ref)
        worst[k] = np.linalg.norm(grads[k] - g_ref) / denom if denom > 0 else 0.0
    bad = {k: v for k, v in worst.items() if v > 2e-2}
    assert not bad, sorted(bad.items(), key=lambda kv: -kv[1])[:5]
