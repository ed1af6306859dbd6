"""Generates tests/golden/loss_curve_smoke.npz: the 200-step history (loss,
learning rate, grad norm) of the CPU restatement of the reference step
(oracle/reference_step.py) on the smoke-parity configuration.

    python tests/golden/make_loss_curve.py [steps]

Data: Zipf(s=1.1) token ids from seed 0 in one shard, read through the
shuffled-epoch stream with stream seed 1 (trainer seed 0 + 1, as the
reference trainer does); parameters from init_params(seed 0). The GPU test
replays the same batches through the B200 step and compares the curves.
"""

from __future__ import annotations

import pathlib
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "gpt-speedrun-tpu_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from oracle import reference_step as ref  # noqa: E402
from rig_b200.config import load_config  # noqa: E402
from rig_b200.tokens import ShardedTokens, ShuffledEpochBatchStream, zipf_tokens  # noqa: E402


def smoke_batches(cfg, steps: int):
    shard = zipf_tokens(steps * cfg.batch_size * (cfg.seq_len + 1) + 17, cfg.vocab_size, 0)
    stream = ShuffledEpochBatchStream(ShardedTokens([shard]), global_batch_size=cfg.batch_size,
                                      seq_len=cfg.seq_len, vocab_size=cfg.vocab_size, seed=1)
    return [stream.next_batch() for _ in range(steps)]


def main(steps: int = 200) -> None:
    torch.set_num_threads(8)
    cfg = load_config("smoke_parity").replace(steps=steps, warmup_steps=int(steps * 0.1 + 0.5))
    trainer = ref.OracleTrainer(cfg, ref.init_params(cfg, 0))
    t0 = time.time()
    for i, (x, y) in enumerate(smoke_batches(cfg, steps)):
        loss = trainer.train_step(x, y)
        if i % 20 == 0:
            print(f"step {i + 1}: loss {loss:.5f} ({time.time() - t0:.0f}s)", flush=True)
    out = pathlib.Path(__file__).resolve().parent / "loss_curve_smoke.npz"
    np.savez_compressed(out, history=np.asarray(trainer.history, dtype=np.float64), steps=steps)
    print("wrote", out)


if __name__ == "__main__":
    main(int(sys.argv[1]) if len(sys.argv) > 1 else 200)
