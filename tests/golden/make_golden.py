"""Generates tests/golden/*.npz by running the REFERENCE implementation.

Run from the repository root in a container where the reference project is
importable (its numpy-only modules; JAX is not needed):

    python tests/golden/make_golden.py /path/to/GPT-speedrun-TPU

It imports the reference's rig/tokens.py and records, for fixed inputs, the
outputs the B200 data loader must reproduce bit for bit: SplitMix64 values,
bounded Feistel permutations and whole distributed batches of
ShuffledEpochBatchStream across ranks, epochs and seeds. The fixtures are
committed; the tests read only the .npz files.
"""

from __future__ import annotations

import pathlib
import sys

import numpy as np


def main(reference_root: str) -> None:
    sys.path.insert(0, reference_root)
    from rig import tokens as rt  # the reference module

    out = pathlib.Path(__file__).resolve().parent
    rng = np.random.default_rng(20240520)

    values = rng.integers(0, 2**63, size=64, dtype=np.uint64)
    values = np.concatenate([values, np.array([0, 1, 2**64 - 1, 0x9E3779B97F4A7C15], np.uint64)])
    mixed = np.array([rt._mix_uint64(int(v)) for v in values], dtype=np.uint64)

    perm_cases = []
    for size in (1, 2, 3, 5, 17, 79, 1000, 123457, 2**20 + 7):
        key = int(rng.integers(0, 2**63))
        idx = np.unique(np.concatenate([np.arange(min(size, 50)), rng.integers(0, size, 50)]))
        perm = np.array([rt._permute_bounded(int(i), size, key) for i in idx], dtype=np.int64)
        perm_cases.append((size, key, idx.astype(np.int64), perm))

    np.savez_compressed(
        out / "tokens_hash.npz",
        mix_in=values, mix_out=mixed,
        perm_sizes=np.array([c[0] for c in perm_cases], np.int64),
        perm_keys=np.array([c[1] for c in perm_cases], np.uint64),
        **{f"perm_idx_{i}": c[2] for i, c in enumerate(perm_cases)},
        **{f"perm_out_{i}": c[3] for i, c in enumerate(perm_cases)},
    )

    # Distributed shuffled stream over ragged uint16 shards (values < vocab).
    vocab = 50304
    lengths = [4097, 10000, 2053, 7777, 513]
    shards = [rng.integers(0, vocab, size=n, dtype=np.uint16) for n in lengths]
    streams = {}
    for seed in (0, 3, 2**40 + 11):
        for world in (1, 2, 4):
            for rank in range(world):
                s = rt.ShuffledEpochBatchStream(
                    rt.ShardedTokens(shards), global_batch_size=8, seq_len=64,
                    vocab_size=vocab, seed=seed, process_index=rank, process_count=world)
                xs, ys = [], []
                for _ in range(60):  # > 1 epoch: 376 windows per epoch / 8 per batch
                    x, y = s.next_batch()
                    xs.append(x)
                    ys.append(y)
                streams[f"x_s{seed}_w{world}_r{rank}"] = np.stack(xs)
                streams[f"y_s{seed}_w{world}_r{rank}"] = np.stack(ys)
    np.savez_compressed(
        out / "tokens_stream.npz",
        **{f"shard_{i}": s for i, s in enumerate(shards)},
        **streams,
    )
    # ShardedTokens.sample (random windows, rig/tokens.py:81-105) and
    # ShardedTokens.sequential (:107-124) over the same ragged shards plus a
    # shard too short to hold a window.
    short = rng.integers(0, vocab, size=40, dtype=np.uint16)
    split = rt.ShardedTokens(shards + [short])
    sampled = {"short_shard": short}
    for seed, (batch, seq) in enumerate([(8, 64), (33, 100), (5, 2000), (1, 4096)]):
        draw = np.random.default_rng(1000 + seed)
        sampled[f"sample_{seed}"] = np.stack([split.sample(draw, batch, seq) for _ in range(4)])
        sampled[f"sample_shape_{seed}"] = np.array([batch, seq], np.int64)
    for i, (index, batch, seq) in enumerate([(0, 8, 64), (5, 8, 64), (1000, 3, 500),
                                             (7, 16, 1000)]):
        sampled[f"seq_{i}"] = split.sequential(index, batch, seq)
        sampled[f"seq_args_{i}"] = np.array([index, batch, seq], np.int64)
    np.savez_compressed(out / "tokens_sample.npz", **sampled)
    print("wrote", out / "tokens_hash.npz", out / "tokens_stream.npz", out / "tokens_sample.npz")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <path of the reference checkout>")
    main(sys.argv[1])
