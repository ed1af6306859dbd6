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


def _tpp_document(tpp=20.0, **model_extra):
    """A schema-6 document shaped like the reference's official recipe: fixed
    tokens-per-parameter horizon, 60m base tier, an untied 125m tier."""

    geom = dict(normalization="rms_norm", position_encoding="rope_base_10000",
                mlp_activation="gelu", vocab_size=50304, semantic_vocab_size=50304, mlp_mult=4)
    return {
        "schema_version": 6,
        "family": {
            "default_tier": "125m", "default_context": "1k",
            "contexts": {"1k": {"seq_len": 1024, "reference_batch_size": 128,
                                "document_masking": False}},
            "parameterization": {"name": "completep_fixed_tpp_v1", "base_tier": "60m",
                                 "depth_alpha": 1.0, "init_std": 0.02,
                                 "attention_scale": "inverse_head_dim", "embeddings": "untied"},
            "tiers": {"60m": {"model": dict(layers=12, heads=6, d_model=384, **geom)},
                      "125m": {"model": dict(layers=12, heads=10, d_model=640, **geom,
                                             **model_extra)}},
        },
        "run": {
            "training": {"duration": {"tokens_per_parameter": tpp}, "dtype": "bfloat16",
                         "sampling": "shuffled_epochs"},
            "kernels": {"vocab_tile_size": 2048},
            "optimizer": {"learning_rate": 2 ** -8, "min_lr_ratio": 0.1, "warmup_ratio": 0.1,
                          "weight_decay": 0.1, "adam_epsilon": 1e-8, "beta1": 0.9,
                          "beta2": 0.95, "grad_clip": 0.0},
        },
    }


def test_fixed_tpp_horizon():
    """steps = floor(tpp_parameters * TPP / tokens_per_step + 0.5) and
    data_multiplier = tpp_parameters / base tier's (train.py:745-751, 792-800)."""

    from rig_b200.config import resolve_config, tpp_parameters

    c = resolve_config(_tpp_document())
    assert c.declared_parameters == 123_456_640  # the reference's 125m tier count
    assert tpp_parameters(_tpp_document()["family"]["tiers"]["60m"]["model"]) == 59_918_208
    assert c.steps == 18838  # 123,456,640 * 20 / 131,072 = 18838.1
    assert c.warmup_steps == 1884
    assert c.data_multiplier == pytest.approx(123_456_640 / 59_918_208)
    assert c.tokens_per_parameter == pytest.approx(18838 * 131072 / 123_456_640)
    # a --tokens-per-parameter style override and a smaller batch
    c2 = resolve_config(_tpp_document(), tokens_per_parameter=1.0, batch_size=8)
    assert c2.steps == int(123_456_640 / 8192 + 0.5) and c2.batch_multiplier == 8 / 128
    with pytest.raises(ValueError):
        resolve_config(_tpp_document(tpp=-1.0))
    with pytest.raises(ValueError):
        load_config("smoke_parity", tokens_per_parameter=20.0)


def test_routed_tier_rules():
    from rig_b200.config import resolve_config

    ok = resolve_config(_tpp_document(experts=6, expert_top_k=2, expert_mult=2))
    assert ok.experts == 6
    for bad in (dict(experts=8, expert_top_k=2, expert_mult=3),   # 2 * 3 != mlp_mult 4
                dict(experts=1, expert_top_k=2, expert_mult=2),   # top_k > experts
                dict(experts=32, expert_top_k=2, expert_mult=2)):  # beyond the kernels
        with pytest.raises(ValueError):
            resolve_config(_tpp_document(**bad))
