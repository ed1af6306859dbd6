"""Pins the CPU restatement (oracle/) with the reference's own known answers:
parameter counts (tests/test_trainer_static.py:153-221), RoPE invariants
(:169-181), CompleteP multipliers (:223-285), and the LCE semantics of
tests/test_linear_cross_entropy.py (dense agreement, invalid targets, zero
gradient on storage rows)."""

import math
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import reference_step as ref
from rig_b200.config import load_config, tensor_multipliers


def _cfg(**kw):
    base = dict(layers=2, heads=2, d_model=64, mlp_mult=4, vocab_size=256, semantic_vocab_size=256,
                parameterization="standard", base_width=64, base_depth=2, depth_alpha=0.0,
                init_std=0.02, attention_scale="inverse_sqrt_head_dim", embeddings="tied")
    base.update(kw)
    return SimpleNamespace(**base)


def _count(p):
    return sum(v.size for v in p.values())


def test_smoke_parameter_count():
    assert _count(ref.init_params(_cfg(), 7)) == 116_160


@pytest.mark.parametrize("tier,expected", [
    ((12, 384, 6), 59_918_208), ((12, 640, 10), 123_456_640), ((16, 896, 14), 244_444_032)])
def test_tier_parameter_counts(tier, expected):
    layers, width, heads = tier
    cfg = _cfg(layers=layers, d_model=width, heads=heads, vocab_size=50304,
               semantic_vocab_size=50304, embeddings="untied", base_width=384, base_depth=12,
               parameterization="completep_fixed_tpp_v1", depth_alpha=1.0)
    # counting only: shapes from the restatement without drawing 100M normals
    d, h = width, 4 * width
    per_block = 12 * d * d + 11 * d
    assert layers * per_block + 2 * 50304 * d + d == expected


def test_baseline_parameter_count():
    cfg = load_config("baseline_125m")
    p = ref.init_params(cfg, 3)
    assert _count(p) == 123_670_272


def test_rope_invariants():
    values = torch.arange(24, dtype=torch.float32).reshape(1, 3, 2, 4)
    rotated = ref.apply_rotary(values)
    assert torch.allclose(rotated[:, 0], values[:, 0], atol=1e-6)
    assert torch.allclose((rotated * rotated).sum(-1), (values * values).sum(-1), rtol=1e-6, atol=1e-5)


def test_completep_multipliers_match_reference_test():
    # tests/test_trainer_static.py:223-285: 250m tier against the 60m base.
    cfg = SimpleNamespace(parameterization="completep_fixed_tpp_v1", d_model=896, base_width=384,
                          layers=16, base_depth=12, depth_alpha=1.0)
    width, depth = 896 / 384, 16 / 12
    lr, eps, wd, _ = ref.multipliers("token_embedding", cfg)
    assert (lr, eps) == pytest.approx((1.0, width ** -1))
    lr, eps, wd, _ = ref.multipliers("blocks/0/qkv_w", cfg)
    assert (lr, eps, wd) == pytest.approx((width ** -1, width ** -1 * depth ** -1, width))
    lr, _, _, _ = ref.multipliers("blocks/0/qkv_b", cfg)
    assert lr == pytest.approx(1.0)
    lr, eps, wd, _ = ref.multipliers("output_embedding", cfg)
    assert (lr, eps, wd) == pytest.approx((width ** -1, 1.0, width))
    # the product's host policy agrees with the restatement everywhere
    full = load_config("baseline_125m")
    for name in ("blocks/3/qkv_w", "blocks/3/ln1_scale", "blocks/0/mlp_up_b", "token_embedding",
                 "final_ln_scale"):
        leaf = name.rsplit("/", 1)[-1]
        assert tensor_multipliers(leaf, name.startswith("blocks/"), full) == pytest.approx(
            ref.multipliers(name, full)[:3])


def _dense_losses(h, e, t, sv):
    logits = h.float() @ e[:sv].float().T
    return -torch.log_softmax(logits, -1).gather(-1, t.long()[:, None])[:, 0]


def test_lce_matches_dense_and_semantics():
    g = torch.Generator().manual_seed(0)
    n, d, v, sv = 64, 32, 259, 250
    h = torch.randn(n, d, generator=g)
    e = torch.randn(v, d, generator=g)
    t = torch.randint(0, sv, (n,), generator=g)
    t[5] = -1
    t[9] = sv + 1
    hh, ee = h.clone().requires_grad_(True), e.clone().requires_grad_(True)
    losses = ref.TiledLinearCrossEntropy.apply(hh, ee, t, sv, torch.float32)
    ok = torch.ones(n, dtype=torch.bool)
    ok[5] = ok[9] = False
    assert torch.isinf(losses[~ok]).all()
    dense = _dense_losses(h[ok], e, t[ok], sv)
    assert torch.allclose(losses[ok], dense, rtol=2e-6, atol=2e-6)
    losses[ok].sum().backward()
    assert torch.count_nonzero(ee.grad[sv:]) == 0
    assert torch.count_nonzero(hh.grad[~ok]) == 0
    hd, ed = h[ok].clone().requires_grad_(True), e.clone().requires_grad_(True)
    _dense_losses(hd, ed, t[ok], sv).sum().backward()
    assert torch.allclose(hh.grad[ok], hd.grad, rtol=3e-6, atol=3e-6)
    assert torch.allclose(ee.grad, ed.grad, rtol=3e-6, atol=3e-6)


def test_learning_rate_schedule():
    cfg = load_config("baseline_125m")
    assert cfg.warmup_steps == 20
    assert ref.learning_rate(1, cfg) == pytest.approx(2 ** -8 / 20, rel=1e-6)
    assert ref.learning_rate(20, cfg) == pytest.approx(2 ** -8, rel=1e-6)
    assert ref.learning_rate(200, cfg) == pytest.approx(0.1 * 2 ** -8, rel=1e-5)


def test_oracle_eval_step_is_masked_loss_sum():
    """train.py:1494-1525 restated: with an all-ones mask the loss sum over the
    token count is the training loss."""

    from rig_b200.model import init_params as b200_init

    cfg = load_config("smoke_parity").replace(batch_size=2, seq_len=32)
    params = b200_init(cfg, 0)
    rng = np.random.default_rng(3)
    x = rng.integers(0, cfg.vocab_size, (2, 32), dtype=np.int32)
    y = rng.integers(0, cfg.vocab_size, (2, 32), dtype=np.int32)
    s, n = ref.eval_step(params, x, y, np.ones((2, 32), np.float32), cfg)
    loss, _ = ref.loss_and_grads(params, x, y, cfg)
    assert n == 64.0
    assert abs(s / n - loss) < 1e-5 * abs(loss)
    s2, n2 = ref.eval_step(params, x, y, np.zeros((2, 32), np.float32), cfg)
    assert s2 == 0.0 and n2 == 0.0


def test_document_segments_golden():
    """tests/test_attention.py:206-211 of the reference (known answer)."""

    tokens = np.asarray([[9, 1, 2, 9, 3], [4, 9, 5, 9, 9]], np.int32)
    np.testing.assert_array_equal(ref.document_segments(tokens, 9),
                                  np.asarray([[1, 1, 1, 2, 2], [0, 1, 1, 2, 3]], np.int32))


def test_segment_attention_is_blockwise_causal():
    """With segments, each document attends as if it were its own sequence."""

    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 2, 12, 8, generator=g) for _ in range(3))
    seg = np.asarray([[0] * 5 + [1] * 7], np.int32)
    out = ref.causal_attention(q, k, v, 0.3, seg)
    a = ref.causal_attention(q[:, :, :5], k[:, :, :5], v[:, :, :5], 0.3)
    b = ref.causal_attention(q[:, :, 5:], k[:, :, 5:], v[:, :, 5:], 0.3)
    torch.testing.assert_close(out, torch.cat([a, b], dim=2))
