"""Run artifacts in the rig's formats: `checkpoint.npz` (rig/runlog.py:96-115)
and `training.riglog` (rig/runlog.py:132-156, 230-301), so the rig's report and
verification tools read a B200 run like one of their own.

* The checkpoint holds every parameter as an fp32 array under the key
  `params/<path>` (the nested parameter tree flattened with mapping keys in
  sorted order and list entries by index, rig/nn.py:63-77), plus the model
  description as UTF-8 JSON bytes under `metadata.json`; it is written to a
  temporary file, fsynced and renamed, so a reader never sees a partial file.
* The training log has three `overall` columns, `train_loss`,
  `learning_rate`, `grad_norm`, plus, for a routed (MoE) model, the router
  statistics columns: one record per optimizer step 1..final_step, exactly the
  rows of the on-device histories the AdamW and router kernels fill.
"""

from __future__ import annotations

import json
import os
import pathlib
from typing import Any, Mapping, Sequence

import numpy as np

from . import logpack

CHECKPOINT_NAME = "checkpoint.npz"
TRAINING_LOG_NAME = f"training{logpack.SUFFIX}"


def flatten_arrays(tree: Any, prefix: str = "params") -> dict[str, np.ndarray]:
    """Flattens a nested parameter tree to `prefix/key/...` names (sorted
    mapping keys, list positions as indices)."""

    flat: dict[str, np.ndarray] = {}

    def walk(node: Any, path: str) -> None:
        if isinstance(node, Mapping):
            for key in sorted(node):
                walk(node[key], f"{path}/{key}")
        elif isinstance(node, (list, tuple)):
            for i, child in enumerate(node):
                walk(child, f"{path}/{i}")
        else:
            flat[path] = np.asarray(node)

    walk(tree, prefix)
    return flat


def nest_params(flat: Mapping[str, np.ndarray], layers: int) -> dict[str, Any]:
    """The reference's parameter tree from this package's `blocks/<b>/<leaf>`
    names: {"blocks": [one dict per block], other tensors at the top level}."""

    tree: dict[str, Any] = {"blocks": [dict() for _ in range(layers)]}
    for name, value in flat.items():
        parts = name.split("/")
        if parts[0] == "blocks":
            tree["blocks"][int(parts[1])][parts[2]] = np.asarray(value, dtype=np.float32)
        else:
            tree[name] = np.asarray(value, dtype=np.float32)
    return tree


def _atomic_write(dest: pathlib.Path, write) -> None:
    """Runs write(binary file) into a temporary file beside `dest`, flushes it
    to disk, then renames it over `dest` (and syncs the directory entry), so a
    reader sees either the old file or the complete new one."""

    import tempfile

    dest = pathlib.Path(dest)
    fd, tmp_name = tempfile.mkstemp(prefix=f".{dest.name}.", suffix=".partial", dir=dest.parent)
    try:
        with os.fdopen(fd, "wb") as fh:
            write(fh)
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(tmp_name, dest)
    except BaseException:
        if os.path.exists(tmp_name):
            os.unlink(tmp_name)
        raise
    dir_fd = os.open(dest.parent, os.O_RDONLY)
    try:
        os.fsync(dir_fd)
    finally:
        os.close(dir_fd)


def save_checkpoint(output_dir: pathlib.Path, params: Any, metadata: Mapping[str, Any]) -> None:
    """checkpoint.npz in `output_dir`: the flattened fp32 parameters under
    `params/...` plus `metadata.json` (UTF-8 JSON with sorted keys, stored as
    uint8), the archive layout of rig/runlog.py:96-115."""

    output_dir = pathlib.Path(output_dir)
    output_dir.mkdir(parents=True, exist_ok=True)
    entries = flatten_arrays(params)
    blob = json.dumps(metadata, sort_keys=True).encode("utf-8")
    entries["metadata.json"] = np.frombuffer(blob, dtype=np.uint8)
    _atomic_write(output_dir / CHECKPOINT_NAME, lambda fh: np.savez(fh, **entries))


def load_checkpoint(path: pathlib.Path) -> tuple[dict[str, np.ndarray], dict[str, Any]]:
    """(flat `blocks/<b>/<leaf>` parameters, metadata) from a checkpoint.npz."""

    with np.load(pathlib.Path(path)) as z:
        meta = json.loads(bytes(z["metadata.json"]).decode("utf-8"))
        flat = {k[len("params/"):]: z[k] for k in z.files if k.startswith("params/")}
    return flat, meta


ROUTER_SUMMARY_METRICS = ("router.entropy", "router.top1_gate", "router.logit_rms")


def training_log_columns(routing_layers: int = 0, experts: int = 0) -> tuple[logpack.Column, ...]:
    """The per-step columns in the order of the history rows
    (rig/runlog.py:133-174): loss, learning rate, gradient norm; a routed run
    appends the balance loss, the max / min expert load and the three router
    summaries averaged over layers, then per layer its three summaries and its
    per-expert load vector (scope "expert", indexed by expert)."""

    cols = [logpack.column("train_loss"), logpack.column("learning_rate"),
            logpack.column("grad_norm")]
    if not routing_layers:
        return tuple(cols)
    cols += [logpack.column("router.balance_loss"), logpack.column("router.max_load"),
             logpack.column("router.min_load")]
    cols += [logpack.column(name) for name in ROUTER_SUMMARY_METRICS]
    for layer in range(routing_layers):
        cols += [logpack.column(name, "block", layer) for name in ROUTER_SUMMARY_METRICS]
        cols += [logpack.column("router.load", "expert", layer, index=e) for e in range(experts)]
    return tuple(cols)


def write_training_log(output_dir: pathlib.Path, history: np.ndarray, *, tokens_per_step: int,
                       final_step: int, flops_per_token: float | None = None,
                       columns: Sequence[logpack.Column] | None = None) -> None:
    """Writes the whole per-step history (rows 1..final_step) atomically."""

    history = np.asarray(history, dtype=np.float32)
    if history.shape[0] > final_step:
        history = history[:final_step]
    cols = tuple(training_log_columns() if columns is None else columns)
    if history.shape != (final_step, len(cols)):
        raise ValueError(f"training history has shape {history.shape}; "
                         f"expected {(final_step, len(cols))}")
    if flops_per_token is not None and flops_per_token <= 0:
        raise ValueError("flops_per_token must be positive when provided")
    output_dir = pathlib.Path(output_dir)
    output_dir.mkdir(parents=True, exist_ok=True)
    dest = output_dir / TRAINING_LOG_NAME
    tmp = output_dir / f".{TRAINING_LOG_NAME}.tmp"
    with logpack.LogWriter(tmp, cols, tokens_per_step=tokens_per_step,
                           flops_per_token=float(flops_per_token or 1.0)) as w:
        for step, row in enumerate(history, 1):
            w.append(step, row)
    os.replace(tmp, dest)


def checkpoint_metadata(config: Any, seed: int) -> dict[str, Any]:
    """The model description that travels in checkpoint.npz, with the key
    structure of recipes/reference/train.py:1042-1076."""

    return {
        "schema_version": 6,
        "seed": int(seed),
        "configuration": {
            "resolved": {
                "training": {"steps": config.steps, "batch_size": config.batch_size,
                             "seq_len": config.seq_len, "dtype": config.dtype_name},
                "kernels": {"attention_backend": "b200_tcgen05_flash",
                            "loss_backend": "tiled", "vocab_tile_size": config.vocab_tile_size},
            },
        },
        "model": {
            "vocab_size": config.vocab_size,
            "semantic_vocab_size": config.semantic_vocab_size,
            "seq_len": config.seq_len,
            "layers": config.layers,
            "heads": config.heads,
            "d_model": config.d_model,
            "mlp_mult": config.mlp_mult,
            "normalization": config.normalization,
            "position_encoding": config.position_encoding,
            "mlp_activation": config.mlp_activation,
            "dtype": config.dtype_name,
            "attention_backend": "b200_tcgen05_flash",
            "loss_backend": "tiled",
            "vocab_tile_size": config.vocab_tile_size,
            "tied_embeddings": bool(config.tied),
            "tier": config.tier,
            "parameterization": config.parameterization,
        },
    }
