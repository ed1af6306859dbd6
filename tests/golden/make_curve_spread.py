"""Generates tests/golden/loss_curve_spread.npz: how far the CPU restatement
of the reference step (oracle/reference_step.py) moves away from its own
200-step smoke history (loss_curve_smoke.npz) under perturbations far below
any implementation difference:

  bf16_ulp  one parameter element (token_embedding[0, 0]) moved to the next
            bfloat16 value (the compute copy of the weights is bf16, so a
            smaller change would not reach the forward pass)
  threads   the same run with one CPU thread (matmul partial sums in another order)

The spread of these runs measures how chaotic the trajectory is; the GPU
curve test compares its own deviation with it.

    python tests/golden/make_curve_spread.py
"""

from __future__ import annotations

import pathlib
import sys

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "gpt-speedrun-tpu_b200"))
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(pathlib.Path(__file__).resolve().parent))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from make_loss_curve import smoke_batches  # noqa: E402
from oracle import reference_step as ref  # noqa: E402
from rig_b200.config import load_config  # noqa: E402


def run(cfg, params, threads: int) -> np.ndarray:
    torch.set_num_threads(threads)
    trainer = ref.OracleTrainer(cfg, params)
    for x, y in smoke_batches(cfg, cfg.steps):
        trainer.train_step(x, y)
    return np.asarray(trainer.history, dtype=np.float64)


def main(steps: int = 200) -> None:
    cfg = load_config("smoke_parity").replace(steps=steps, warmup_steps=int(steps * 0.1 + 0.5))
    params = ref.init_params(cfg, 0)
    bumped = {k: v.copy() for k, v in params.items()}
    e = bumped["token_embedding"]
    b16 = torch.tensor(float(e[0, 0])).bfloat16()
    e[0, 0] = float(torch.nextafter(b16, torch.tensor(1.0, dtype=torch.bfloat16)).float())
    out = {"bf16_ulp": run(cfg, bumped, 8), "threads": run(cfg, params, 1)}
    path = pathlib.Path(__file__).resolve().parent / "loss_curve_spread.npz"
    np.savez_compressed(path, steps=steps, **out)
    print("wrote", path)


if __name__ == "__main__":
    main(int(sys.argv[1]) if len(sys.argv) > 1 else 200)
