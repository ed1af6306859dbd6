"""Run artifacts in the rig's formats (rig/runlog.py:96-156, rig/logpack.py):
the training log is byte-identical to what the reference's own writer produces
for the same history (fixture written by tests/golden/make_artifacts.py), and
checkpoint.npz has the reference's key layout and round-trips."""

import json
import pathlib

import numpy as np
import pytest

from rig_b200 import logpack, runlog
from rig_b200.config import load_config
from rig_b200.model import init_params

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def _maker():
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_artifacts", GOLDEN / "make_artifacts.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _history():
    return _maker().history()


def test_registry_ids_match_reference():
    ids = json.loads((GOLDEN / "riglog_ids.json").read_text())
    for name, value in ids.items():
        if name.startswith("scope."):
            assert logpack.SCOPE_IDS[name[len("scope."):]][0] == value, name
        else:
            assert logpack.METRIC_IDS[name] == value, name


def test_routed_training_log_bytes_match_reference_writer(tmp_path):
    """A routed model's log: the router statistics columns after the dense
    three, per layer the summaries and the per-expert load (scope "expert")."""

    mk = _maker()
    cols = runlog.training_log_columns(mk.MOE_LAYERS, mk.MOE_EXPERTS)
    assert len(cols) == 3 + 6 + mk.MOE_LAYERS * (3 + mk.MOE_EXPERTS)
    runlog.write_training_log(tmp_path, mk.moe_history(), tokens_per_step=4096, final_step=20,
                              flops_per_token=987654321.0, columns=cols)
    ours = (tmp_path / runlog.TRAINING_LOG_NAME).read_bytes()
    assert ours == (GOLDEN / "training_moe.riglog").read_bytes()
    log = logpack.read_log(GOLDEN / "training_moe.riglog")
    assert log.columns == cols
    loads = [c for c in log.columns if c.scope_id == logpack.SCOPE_IDS["expert"][0]]
    assert [(c.layer, c.index) for c in loads] == [(l, e) for l in range(mk.MOE_LAYERS)
                                                  for e in range(mk.MOE_EXPERTS)]


def test_column_scope_rules():
    with pytest.raises(ValueError):
        logpack.column("router.load", "expert", 0)  # expert scope needs an index
    with pytest.raises(ValueError):
        logpack.column("router.entropy", "block", 0, index=1)
    with pytest.raises(ValueError):
        logpack.column("router.entropy", "block")
    with pytest.raises(KeyError):
        logpack.column("router.unknown")


def test_training_log_bytes_match_reference_writer(tmp_path):
    h = _history()
    runlog.write_training_log(tmp_path, h, tokens_per_step=2048, final_step=20,
                              flops_per_token=123456789.0)
    ours = (tmp_path / runlog.TRAINING_LOG_NAME).read_bytes()
    assert ours == (GOLDEN / "training_smoke.riglog").read_bytes()


def test_read_reference_log():
    log = logpack.read_log(GOLDEN / "training_smoke.riglog")
    assert log.tokens_per_step == 2048 and log.flops_per_token == 123456789.0
    assert [c.metric_id for c in log.columns] == [4, 5, 6]
    assert all(c.scope_id == 1 and c.layer == -1 and c.index == -1 for c in log.columns)
    assert log.steps.tolist() == list(range(1, 21))
    np.testing.assert_array_equal(log.values, _history())


def test_partial_record_is_dropped(tmp_path):
    raw = (GOLDEN / "training_smoke.riglog").read_bytes()
    (tmp_path / "cut.riglog").write_bytes(raw[:-5])
    log = logpack.read_log(tmp_path / "cut.riglog")
    assert log.steps.tolist() == list(range(1, 20))


def test_training_log_rejects_wrong_width(tmp_path):
    with pytest.raises(ValueError):
        runlog.write_training_log(tmp_path, np.zeros((5, 2), np.float32), tokens_per_step=1,
                                  final_step=5)
    with pytest.raises(ValueError):
        logpack.LogWriter(tmp_path / "x.riglog", runlog.training_log_columns(),
                          tokens_per_step=0, flops_per_token=1.0)


def test_checkpoint_layout_and_roundtrip(tmp_path):
    cfg = load_config("smoke_parity")
    flat = init_params(cfg, 0)
    tree = runlog.nest_params(flat, cfg.layers)
    meta = runlog.checkpoint_metadata(cfg, 0)
    runlog.save_checkpoint(tmp_path, tree, meta)
    path = tmp_path / runlog.CHECKPOINT_NAME
    with np.load(path) as z:
        keys = list(z.files)
    # rig/nn.py:63-77: mapping keys sorted, list entries by index, "params/" prefix
    block0 = sorted(k for k in flat if k.startswith("blocks/0/"))
    assert keys[: len(block0)] == ["params/" + k for k in block0]
    assert keys[-1] == "metadata.json"
    top = [k for k in keys if not k.startswith("params/blocks/") and k != "metadata.json"]
    assert top == sorted(top) and "params/token_embedding" in top
    loaded, meta2 = runlog.load_checkpoint(path)
    assert meta2 == json.loads(json.dumps(meta, sort_keys=True))
    assert set(loaded) == set(flat)
    for k, v in flat.items():
        assert loaded[k].dtype == np.float32
        np.testing.assert_array_equal(loaded[k], v)
    assert not any(p.name.startswith(".") for p in tmp_path.iterdir())
