"""Evaluation step (recipes/reference/train.py:1494-1525) against the CPU
restatement, and the trainer's run artifacts (checkpoint.npz, training.riglog)
against its own device state."""

import numpy as np
import pytest
import torch

from oracle import reference_step as ref
from rig_b200 import logpack, ops, runlog
from rig_b200.config import load_config
from rig_b200.model import GPTTrainer, init_params
from rig_b200.tokens import zipf_tokens

pytestmark = pytest.mark.gpu


def _batch(cfg, seed):
    b, t = cfg.batch_size, cfg.seq_len
    w = zipf_tokens(b * (t + 1), cfg.vocab_size, seed).astype(np.int32).reshape(b, t + 1)
    return np.ascontiguousarray(w[:, :-1]), np.ascontiguousarray(w[:, 1:])


def test_eval_step_matches_oracle(cuda):
    cfg = load_config("smoke_parity")
    params = init_params(cfg, 0)
    x, y = _batch(cfg, 5)
    mask = (np.random.default_rng(1).random(x.shape) < 0.7).astype(np.float32)
    want_sum, want_count = ref.eval_step(params, x, y, mask, cfg)
    tr = GPTTrainer(cfg, cfg.batch_size, cuda)
    tr.load_params(params)
    out = tr.eval_step(torch.from_numpy(x).to(cuda), torch.from_numpy(y).to(cuda),
                       torch.from_numpy(mask).to(cuda)).cpu().numpy()
    assert ops.device_error() == 0
    assert out[1] == want_count  # exact count (sum of 0/1 in fp32)
    assert abs(out[0] - want_sum) / want_sum < 1e-3, (out[0], want_sum)
    # evaluating leaves the parameters and the optimizer untouched
    assert int(tr.step_dev.item()) == 0
    np.testing.assert_array_equal(tr.export()["blocks/0/qkv_w"], params["blocks/0/qkv_w"])


def test_masked_loss_sum_kernel(cuda):
    g = torch.Generator().manual_seed(0)
    losses = torch.rand(100003, generator=g) * 10
    mask = (torch.rand(100003, generator=g) < 0.5).float()
    out = ops.masked_loss_sum(losses.to(cuda), mask.to(cuda)).cpu()
    assert out[1].item() == mask.sum().item()
    assert abs(out[0].item() - (losses * mask).double().sum().item()) < 1e-5 * out[0].item()
    again = ops.masked_loss_sum(losses.to(cuda), mask.to(cuda)).cpu()
    assert torch.equal(out, again)  # one block, fixed order: bit-identical


def test_checkpoint_and_training_log(cuda, tmp_path):
    cfg = load_config("smoke_parity")
    tr = GPTTrainer(cfg, cfg.batch_size, cuda)
    tr.load_params(init_params(cfg, 0))
    steps = 3
    for s in range(steps):
        x, y = _batch(cfg, 10 + s)
        tr.train_step(torch.from_numpy(x).to(cuda), torch.from_numpy(y).to(cuda))
    torch.cuda.synchronize()
    tr.save_checkpoint(tmp_path, seed=0)
    tr.write_training_log(tmp_path, steps, flops_per_token=1.0e6)
    flat, meta = runlog.load_checkpoint(tmp_path / runlog.CHECKPOINT_NAME)
    want = tr.export()
    assert set(flat) == set(want)
    for k in want:
        np.testing.assert_array_equal(flat[k], want[k])
    assert meta["model"]["layers"] == cfg.layers and meta["seed"] == 0
    log = logpack.read_log(tmp_path / runlog.TRAINING_LOG_NAME)
    assert log.steps.tolist() == [1, 2, 3]
    np.testing.assert_array_equal(log.values, tr.history[:steps].cpu().numpy())
    assert log.tokens_per_step == cfg.batch_size * cfg.seq_len
    # a trainer restored from the checkpoint computes the same forward loss
    tr2 = GPTTrainer(cfg, cfg.batch_size, cuda)
    tr2.load_params(flat)
    x, y = _batch(cfg, 99)
    for t in (tr, tr2):
        t.set_batch(torch.from_numpy(x).to(cuda), torch.from_numpy(y).to(cuda))
        t.forward()
    assert tr.loss.item() == tr2.loss.item()
