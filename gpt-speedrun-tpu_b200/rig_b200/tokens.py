"""Token shards and the deterministic distributed batch stream.

Same API and bit-exact output as the reference's rig/tokens.py:
`ShardedTokens` (:70-124), the SplitMix64/Feistel helpers (:127-168),
`ShuffledEpochBatchStream` (:171-272) and `load_token_file` (:333-372). The
per-row permutation + window copy runs in native code
(`gptb200_gather_windows`, csrc/tokens.cpp) for uint16 shards; only the
once-per-epoch shard order uses numpy's PCG64 (`default_rng(SeedSequence(
(seed lo, seed hi, epoch lo, epoch hi)))`, :222-236), exactly as the reference.

Also here: the llm.c shard writer and the seeded Zipf token generator used for
the synthetic benchmark data.
"""

from __future__ import annotations

import ctypes
import hashlib
import pathlib
from typing import Sequence

import numpy as np

from . import _lib

_UINT64_MASK = (1 << 64) - 1
LLMC_MAGIC = 20240520


def mix_uint64(value: int) -> int:
    return int(_lib.load().gptb200_mix_uint64(ctypes.c_uint64(value & _UINT64_MASK)))


def permute_bounded(value: int, size: int, key: int) -> int:
    if not 0 <= value < size:
        raise ValueError("permutation input must lie inside its domain")
    return int(_lib.load().gptb200_permute_bounded(value, size, key & _UINT64_MASK))


class ShardedTokens:
    """A logical token stream backed by one or more (memory-mapped) shards."""

    def __init__(self, shards: Sequence[np.ndarray]) -> None:
        self.shards = tuple(shards)
        if not self.shards:
            raise ValueError("a token split must contain at least one shard")

    def __len__(self) -> int:
        return sum(len(s) for s in self.shards)

    def sample(self, rng: np.random.Generator, batch_size: int, seq_len: int) -> np.ndarray:
        """Random windows, identical draws to rig/tokens.py:81-105."""

        valid_starts = np.asarray([max(0, len(s) - seq_len) for s in self.shards], dtype=np.int64)
        total = int(valid_starts.sum())
        if total <= 0:
            raise ValueError("no shard is long enough for seq_len + 1")
        choices = rng.choice(len(self.shards), size=batch_size, p=valid_starts / total)
        windows = np.empty((batch_size, seq_len + 1), dtype=np.int32)
        offsets = np.arange(seq_len + 1)
        for shard_index in np.unique(choices):
            rows = np.flatnonzero(choices == shard_index)
            shard = self.shards[int(shard_index)]
            starts = rng.integers(0, len(shard) - seq_len, size=len(rows))
            windows[rows] = shard[starts[:, None] + offsets]
        return windows


class ShuffledEpochBatchStream:
    """Deterministic, distributed, no-replacement windows within each epoch."""

    def __init__(self, tokens: ShardedTokens, *, global_batch_size: int, seq_len: int,
                 vocab_size: int, seed: int, process_index: int = 0,
                 process_count: int = 1) -> None:
        if global_batch_size <= 0 or seq_len <= 0 or vocab_size <= 0:
            raise ValueError("stream batch, sequence, and vocabulary sizes must be positive")
        if process_count <= 0 or not 0 <= process_index < process_count:
            raise ValueError("invalid process index/count for shuffled stream")
        if global_batch_size % process_count:
            raise ValueError("global batch size must be divisible by process count")
        self.tokens = tokens
        self.global_batch_size = int(global_batch_size)
        self.local_batch_size = global_batch_size // process_count
        self.seq_len = int(seq_len)
        self.vocab_size = int(vocab_size)
        self.seed = int(seed) & _UINT64_MASK
        self.process_index = int(process_index)
        self.window_counts = np.asarray(
            [(len(s) - 1) // seq_len for s in tokens.shards], dtype=np.int64)
        self.windows_per_epoch = int(self.window_counts.sum())
        if self.windows_per_epoch <= 0:
            raise ValueError(f"no training shard contains a full {seq_len:,}-target window")
        self._global_cursor = 0
        self._planned_epoch = -1
        self._ordered_shards = np.empty((0,), dtype=np.int64)
        self._ordered_cumulative = np.empty((0,), dtype=np.int64)
        self._epoch_key = 0
        self._native = all(
            isinstance(s, np.ndarray) and s.dtype == np.uint16 and s.ndim == 1
            and s.flags["C_CONTIGUOUS"] for s in tokens.shards)
        if self._native:
            self._ptrs = (ctypes.c_void_p * len(tokens.shards))(
                *[s.ctypes.data for s in tokens.shards])
            self._lengths = np.asarray([len(s) for s in tokens.shards], dtype=np.int64)

    def _prepare_epoch(self, epoch: int) -> None:
        words = (self.seed & 0xFFFFFFFF, self.seed >> 32, epoch & 0xFFFFFFFF, epoch >> 32)
        rng = np.random.default_rng(np.random.SeedSequence(words))
        self._ordered_shards = rng.permutation(len(self.tokens.shards)).astype(np.int64, copy=False)
        self._ordered_cumulative = np.cumsum(self.window_counts[self._ordered_shards], dtype=np.int64)
        self._epoch_key = mix_uint64(self.seed ^ mix_uint64(epoch))
        self._planned_epoch = epoch

    def _rows(self, first_ordinal: int, rows: int, out: np.ndarray) -> None:
        """Fills out[rows, seq_len + 1] with windows of consecutive global ordinals."""

        done = 0
        while done < rows:
            epoch, ordinal = divmod(first_ordinal + done, self.windows_per_epoch)
            if epoch != self._planned_epoch:
                self._prepare_epoch(epoch)
            take = min(rows - done, self.windows_per_epoch - ordinal)
            if self._native:
                status = _lib.load().gptb200_gather_windows(
                    self._ptrs, self._lengths.ctypes.data, self._ordered_shards.ctypes.data,
                    self._ordered_cumulative.ctypes.data, len(self.tokens.shards),
                    self.windows_per_epoch, self._epoch_key, ordinal, take, self.seq_len,
                    self.vocab_size, out[done:].ctypes.data)
                if status not in (0, 5):
                    _lib.check(status, "gptb200_gather_windows")
            else:
                for r in range(take):
                    permuted = permute_bounded(ordinal + r, self.windows_per_epoch, self._epoch_key)
                    oi = int(np.searchsorted(self._ordered_cumulative, permuted, side="right"))
                    prev = int(self._ordered_cumulative[oi - 1]) if oi else 0
                    shard = self.tokens.shards[int(self._ordered_shards[oi])]
                    start = (permuted - prev) * self.seq_len
                    out[done + r] = shard[start : start + self.seq_len + 1]
            done += take

    def next_batch(self) -> tuple[np.ndarray, np.ndarray]:
        rank_start = self._global_cursor + self.process_index * self.local_batch_size
        windows = np.empty((self.local_batch_size, self.seq_len + 1), dtype=np.int32)
        self._rows(rank_start, self.local_batch_size, windows)
        self._global_cursor += self.global_batch_size
        lo, hi = int(windows.min()), int(windows.max())
        if lo < 0 or hi >= self.vocab_size:
            raise ValueError(
                f"streamed token ids [{lo}, {hi}] do not fit vocab_size={self.vocab_size}")
        return np.ascontiguousarray(windows[:, :-1]), np.ascontiguousarray(windows[:, 1:])


# ----------------------------------------------------------------- files
def load_token_file(path: pathlib.Path, raw_dtype: str = "uint16", data_format: str = "auto"):
    """llm.c shard (1024-byte header, magic 20240520, version 1), .npy, or raw."""

    path = pathlib.Path(path).expanduser().resolve()
    if not path.is_file():
        raise FileNotFoundError(f"token data not found: {path}")
    if path.suffix == ".npy":
        values = np.load(path, mmap_mode="r", allow_pickle=False)
        if values.ndim != 1:
            raise ValueError(f"expected a one-dimensional token array in {path}")
        return values
    if path.suffix in (".txt", ".text"):
        return np.frombuffer(path.read_bytes(), dtype=np.uint8)
    with path.open("rb") as handle:
        head = handle.read(1024)
    header = np.frombuffer(head, dtype="<i4", count=256) if len(head) == 1024 else np.empty(0, np.int32)
    is_llmc = len(header) == 256 and int(header[0]) == LLMC_MAGIC
    if data_format == "llmc" and not is_llmc:
        raise ValueError(f"{path} does not have an llm.c FineWeb header")
    if data_format != "raw" and is_llmc:
        if int(header[1]) != 1:
            raise ValueError(f"unsupported llm.c data version {int(header[1])} in {path}")
        count = int(header[2])
        if count <= 0:
            raise ValueError(f"invalid llm.c token count {count} in {path}")
        if path.stat().st_size != 1024 + 2 * count:
            raise ValueError(f"bad llm.c shard size for {path}")
        return np.memmap(path, dtype="<u2", mode="r", offset=1024, shape=(count,))
    dtype = np.dtype(raw_dtype)
    if path.stat().st_size % dtype.itemsize:
        raise ValueError(f"{path} size is not a multiple of dtype {raw_dtype}")
    return np.memmap(path, dtype=dtype, mode="r")


def write_llmc_shard(path: pathlib.Path, tokens: np.ndarray) -> str:
    """Writes uint16 tokens with the llm.c header; returns the file's SHA-256."""

    tokens = np.asarray(tokens)
    if tokens.min() < 0 or tokens.max() > 0xFFFF:
        raise ValueError("llm.c shards hold uint16 token ids")
    header = np.zeros(256, dtype="<i4")
    header[0], header[1], header[2] = LLMC_MAGIC, 1, len(tokens)
    path = pathlib.Path(path)
    with path.open("wb") as handle:
        handle.write(header.tobytes())
        handle.write(tokens.astype("<u2").tobytes())
    return file_sha256(path)


def file_sha256(path: pathlib.Path) -> str:
    digest = hashlib.sha256()
    with pathlib.Path(path).open("rb") as handle:
        for chunk in iter(lambda: handle.read(1 << 20), b""):
            digest.update(chunk)
    return digest.hexdigest()


def zipf_tokens(n: int, vocab: int, seed: int, s: float = 1.1) -> np.ndarray:
    """Bounded Zipf ids: p(k) ∝ k^-s for k = 1..vocab, token id = k - 1."""

    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    p = ranks ** (-s)
    p /= p.sum()
    rng = np.random.default_rng(seed)
    return rng.choice(vocab, size=n, p=p).astype(np.uint16 if vocab <= 65536 else np.int32)
