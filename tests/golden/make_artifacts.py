"""Writes tests/golden/training_smoke.riglog with the reference's own
rig/logpack.py (the training-log columns of rig/runlog.py:132-156) from a fixed
synthetic history, and tests/golden/training_moe.riglog with the routed-model
columns (rig/runlog.py:152-173, restated here in the same order because
rig/runlog.py itself imports jax) for 2 layers x 4 experts, plus the registry
ids they resolve. Run in a checkout where
the reference project is importable (its logpack/metrics modules need only numpy):

    python tests/golden/make_artifacts.py /path/to/GPT-speedrun-TPU
"""

import json
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent


def history() -> np.ndarray:
    rng = np.random.default_rng(7)
    h = np.empty((20, 3), np.float32)
    h[:, 0] = 10.8 - 0.2 * np.arange(20) + 0.01 * rng.standard_normal(20)
    h[:, 1] = np.float32(2.0 ** -8) * np.minimum(1.0, (np.arange(20) + 1) / 2.0)
    h[:, 2] = np.abs(1.0 + rng.standard_normal(20))
    return h


MOE_LAYERS, MOE_EXPERTS = 2, 4
ROUTER_SUMMARY = ("router.entropy", "router.top1_gate", "router.logit_rms")


def moe_history() -> np.ndarray:
    rng = np.random.default_rng(11)
    width = 3 + 6 + MOE_LAYERS * (3 + MOE_EXPERTS)
    h = np.abs(rng.standard_normal((20, width))).astype(np.float32)
    h[:, :3] = history()
    return h


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from rig import logpack, metrics  # noqa: E402  (the reference's modules)

    cols = [logpack.column("train_loss"), logpack.column("learning_rate"),
            logpack.column("grad_norm")]
    out = HERE / "training_smoke.riglog"
    with logpack.LogWriter(out, cols, tokens_per_step=2048, flops_per_token=123456789.0) as w:
        for step, row in enumerate(history(), 1):
            w.append(step, row)
    moe_cols = cols + [logpack.column("router.balance_loss"), logpack.column("router.max_load"),
                       logpack.column("router.min_load")]
    moe_cols += [logpack.column(name) for name in ROUTER_SUMMARY]
    for layer in range(MOE_LAYERS):
        moe_cols += [logpack.column(name, "block", layer) for name in ROUTER_SUMMARY]
        moe_cols += [logpack.column("router.load", "expert", layer, index=e)
                     for e in range(MOE_EXPERTS)]
    moe_out = HERE / "training_moe.riglog"
    with logpack.LogWriter(moe_out, moe_cols, tokens_per_step=4096,
                           flops_per_token=987654321.0) as w:
        for step, row in enumerate(moe_history(), 1):
            w.append(step, row)
    names = ("train_loss", "learning_rate", "grad_norm", "router.balance_loss", "router.max_load",
             "router.min_load", "router.load", *ROUTER_SUMMARY)
    ids = {name: metrics.metric(name).id for name in names}
    for scope in ("overall", "block", "expert"):
        ids["scope." + scope] = metrics.scope(scope).id
    (HERE / "riglog_ids.json").write_text(json.dumps(ids, sort_keys=True) + "\n")
    print(f"wrote {out} ({out.stat().st_size} bytes) and riglog_ids.json")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path of the reference checkout>")
    main(sys.argv[1])
