"""Config resolution mirrors recipes/reference/train.py:688-862."""

import pytest

from rig_b200.config import effective_adam_betas, horizon_scales, learning_rate, load_config


def test_baseline_config():
    c = load_config("baseline_125m")
    assert (c.layers, c.d_model, c.heads, c.head_dim, c.hidden) == (12, 768, 12, 64, 3072)
    assert (c.seq_len, c.batch_size, c.steps, c.warmup_steps) == (1024, 128, 200, 20)
    assert c.tied and c.vocab_size == 50304
    assert c.width_multiplier == 2.0 and c.depth_multiplier == 1.0 and c.branch_scale == 1.0
    assert c.softmax_scale == 1 / 64
    assert effective_adam_betas(c) == (pytest.approx(0.9), pytest.approx(0.95))
    assert horizon_scales(c) == (1.0, 1.0, 1.0)
    assert learning_rate(20, c) == pytest.approx(2 ** -8)


def test_smoke_config_and_batch_override():
    c = load_config("smoke_parity")
    assert (c.layers, c.d_model, c.heads, c.seq_len, c.batch_size) == (4, 256, 4, 256, 8)
    assert c.branch_scale == 0.25
    c2 = load_config("smoke_parity", batch_size=16)
    assert c2.batch_multiplier == 2.0
    b1, b2 = effective_adam_betas(c2)
    assert b1 == pytest.approx(0.8) and b2 == pytest.approx(0.9)
