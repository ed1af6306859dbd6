"""Token shards and the deterministic distributed batch stream.

Public names and results match the reference data loader (rig/tokens.py):
`ShardedTokens` with `sample` (random windows, :81-105) and `sequential`
(:107-124), `ShuffledEpochBatchStream` (:171-272) and `load_token_file`
(:333-372); every batch is bit-identical to the reference's for the same
shards and seeds (pinned by fixtures made from the reference itself).

How it is organised here: the stream keeps only a cursor and, per epoch, the
shard order, which is a draw of numpy's PCG64 Generator seeded with the four
32-bit words (seed lo, seed hi, epoch lo, epoch hi) and therefore stays in
numpy. Everything else of an epoch -- the window table, the epoch key, the
keyed permutation of the window ordinals and the copy into the batch -- runs
in native code over a whole local batch at a time (`gptb200_epoch_windows`,
csrc/tokens.cpp), for shards of any integer element type.

Also here: the llm.c shard writer, a file digest and the seeded Zipf token
generator of the synthetic benchmark data.
"""

from __future__ import annotations

import ctypes
import hashlib
import pathlib
import struct
from typing import Sequence

import numpy as np

from . import _lib

_MASK64 = (1 << 64) - 1
LLMC_MAGIC = 20240520      # llm.c token file: 256 little-endian int32 header words
LLMC_VERSION = 1           # header[0] = magic, header[1] = version, header[2] = count,
LLMC_HEADER_BYTES = 1024   # then `count` little-endian uint16 tokens

# numpy element type -> GPTB200_TOKENS_* code of the native window copy
_DTYPE_CODES = {np.dtype(np.uint8): 0, np.dtype(np.uint16): 1, np.dtype(np.int32): 2,
                np.dtype(np.uint32): 3, np.dtype(np.int64): 4}


def mix_uint64(value: int) -> int:
    """SplitMix64 finaliser of a 64-bit word (rig/tokens.py:127-133)."""

    return int(_lib.load().gptb200_mix_uint64(ctypes.c_uint64(value & _MASK64)))


def permute_bounded(value: int, size: int, key: int) -> int:
    """Image of `value` under the keyed permutation of [0, size) (rig/tokens.py:136-168)."""

    if value < 0 or value >= size:
        raise ValueError(f"{value} is outside the permutation domain [0, {size})")
    return int(_lib.load().gptb200_permute_bounded(value, size, key & _MASK64))


def _native_shard(shard) -> np.ndarray:
    """The shard as a 1-D C-contiguous array of a type the native copy reads."""

    arr = np.asarray(shard)
    if arr.ndim != 1:
        raise ValueError(f"token shards are one-dimensional, got shape {arr.shape}")
    if arr.dtype not in _DTYPE_CODES:
        arr = arr.astype(np.int64)
    return np.ascontiguousarray(arr)


class ShardedTokens:
    """A token split: several 1-D shards read as one logical stream, without
    concatenating them (shards may be memory-mapped files)."""

    def __init__(self, shards: Sequence[np.ndarray]) -> None:
        shards = tuple(shards)
        if len(shards) == 0:
            raise ValueError("ShardedTokens needs at least one shard")
        self.shards = shards
        self.lengths = np.array([len(s) for s in shards], dtype=np.int64)

    def __len__(self) -> int:
        return int(self.lengths.sum())

    def window_counts(self, seq_len: int) -> np.ndarray:
        """Whole (seq_len + 1)-token windows per shard at stride seq_len."""

        return np.maximum(self.lengths - 1, 0) // seq_len

    def sample(self, rng: np.random.Generator, batch_size: int, seq_len: int) -> np.ndarray:
        """`batch_size` random windows of seq_len + 1 tokens (int32).

        Uniform over every start position of every shard: a shard is drawn for
        each row with probability proportional to its number of starts, then,
        shard by shard in increasing index order, the start offsets of that
        shard's rows. The same generator state yields the reference's windows
        (rig/tokens.py:81-105), because the draws are made in the same order.
        """

        starts_per_shard = np.maximum(self.lengths - seq_len, 0)
        total = int(starts_per_shard.sum())
        if total == 0:
            raise ValueError(f"no shard holds seq_len + 1 = {seq_len + 1} tokens "
                             f"({len(self.shards)} shard(s), {len(self)} tokens)")
        picks = rng.choice(len(self.shards), size=batch_size, p=starts_per_shard / total)
        out = np.empty((batch_size, seq_len + 1), dtype=np.int32)
        span = np.arange(seq_len + 1)
        order = np.argsort(picks, kind="stable")
        bounds = np.flatnonzero(np.diff(picks[order])) + 1
        for group in np.split(order, bounds):
            s = int(picks[group[0]])
            first = rng.integers(0, int(self.lengths[s]) - seq_len, size=group.size)
            out[group] = self.shards[s][first[:, None] + span]
        return out

    def sequential(self, batch_index: int, batch_size: int, seq_len: int) -> np.ndarray:
        """Batch `batch_index` of the split read front to back in
        non-overlapping windows (stride seq_len), wrapping around at the end
        (rig/tokens.py:107-124)."""

        counts = self.window_counts(seq_len)
        total = int(counts.sum())
        if total == 0:
            raise ValueError(f"no shard holds a full {seq_len + 1}-token window")
        ends = np.cumsum(counts)
        ordinals = (batch_index * batch_size + np.arange(batch_size, dtype=np.int64)) % total
        which = np.searchsorted(ends, ordinals, side="right")
        out = np.empty((batch_size, seq_len + 1), dtype=np.int32)
        for row, (w, s) in enumerate(zip(ordinals, which)):
            start = (int(w) - (int(ends[s - 1]) if s else 0)) * seq_len
            out[row] = self.shards[int(s)][start : start + seq_len + 1]
        return out


class ShuffledEpochBatchStream:
    """Epoch-by-epoch shuffled windows, split across data-parallel ranks.

    Every epoch visits each whole window of the split exactly once, in an
    order fixed by (seed, epoch); global batch b holds the epoch-order
    windows [b * global_batch_size, (b + 1) * global_batch_size) of the
    running sequence, and rank r takes the r-th contiguous slice of it
    (rig/tokens.py:171-272). `next_batch` returns int32 (inputs, targets),
    the targets shifted by one token.
    """

    def __init__(self, tokens: ShardedTokens, *, global_batch_size: int, seq_len: int,
                 vocab_size: int, seed: int, process_index: int = 0,
                 process_count: int = 1) -> None:
        for name, value in (("global_batch_size", global_batch_size), ("seq_len", seq_len),
                            ("vocab_size", vocab_size), ("process_count", process_count)):
            if value < 1:
                raise ValueError(f"{name} must be at least 1, got {value}")
        if not 0 <= process_index < process_count:
            raise ValueError(f"process_index {process_index} is not a rank of {process_count}")
        if global_batch_size % process_count:
            raise ValueError(f"global_batch_size {global_batch_size} does not split evenly over "
                             f"{process_count} processes")
        self.tokens = tokens
        self.global_batch_size = int(global_batch_size)
        self.local_batch_size = self.global_batch_size // int(process_count)
        self.seq_len = int(seq_len)
        self.vocab_size = int(vocab_size)
        self.seed = int(seed) & _MASK64
        self.process_index = int(process_index)
        self.windows_per_epoch = int(tokens.window_counts(self.seq_len).sum())
        if self.windows_per_epoch == 0:
            raise ValueError(f"no shard holds {self.seq_len} targets plus one input token")
        self._cursor = 0  # global window ordinal of the next global batch
        self._orders: dict[int, np.ndarray] = {}
        arrays = [_native_shard(s) for s in tokens.shards]
        codes = {_DTYPE_CODES[a.dtype] for a in arrays}
        if len(codes) != 1:  # one element type per call of the native copy
            arrays = [a.astype(np.int64) for a in arrays]
            codes = {_DTYPE_CODES[np.dtype(np.int64)]}
        self._arrays = arrays  # keeps converted shards alive
        self._dtype_code = codes.pop()
        self._ptrs = (ctypes.c_void_p * len(arrays))(*[a.ctypes.data for a in arrays])
        self._lengths = np.ascontiguousarray(tokens.lengths)

    def epoch_order(self, epoch: int) -> np.ndarray:
        """Shard visiting order of `epoch`: numpy PCG64 seeded with the 32-bit
        words of the seed and of the epoch (rig/tokens.py:222-227)."""

        order = self._orders.get(epoch)
        if order is None:
            words = (self.seed & 0xFFFFFFFF, self.seed >> 32, epoch & 0xFFFFFFFF, epoch >> 32)
            gen = np.random.default_rng(np.random.SeedSequence(words))
            order = np.ascontiguousarray(gen.permutation(len(self.tokens.shards)), dtype=np.int64)
            self._orders = {epoch: order}  # batches move forward: keep the latest epoch only
        return order

    def _fill(self, first: int, out: np.ndarray) -> None:
        """Windows of global ordinals first .. first + len(out) - 1 into out."""

        lib = _lib.load()
        row = 0
        while row < len(out):
            epoch, start = divmod(first + row, self.windows_per_epoch)
            take = min(len(out) - row, self.windows_per_epoch - start)
            order = self.epoch_order(epoch)
            status = lib.gptb200_epoch_windows(
                self._ptrs, self._lengths.ctypes.data, len(self._arrays), self._dtype_code,
                order.ctypes.data, self.seq_len, self.seed, epoch, start, take, self.vocab_size,
                out[row:].ctypes.data)
            if status != 5:  # GPTB200_ERANGE is reported by next_batch with the ids
                _lib.check(status, "gptb200_epoch_windows")
            row += take

    def next_batch(self) -> tuple[np.ndarray, np.ndarray]:
        windows = np.empty((self.local_batch_size, self.seq_len + 1), dtype=np.int32)
        self._fill(self._cursor + self.process_index * self.local_batch_size, windows)
        self._cursor += self.global_batch_size
        if windows.size and (windows.min() < 0 or windows.max() >= self.vocab_size):
            raise ValueError(f"token ids in [{windows.min()}, {windows.max()}] fall outside "
                             f"the vocabulary of {self.vocab_size}")
        return np.ascontiguousarray(windows[:, :-1]), np.ascontiguousarray(windows[:, 1:])


# ----------------------------------------------------------------- files
def _llmc_header(path: pathlib.Path) -> tuple[int, ...] | None:
    """The 256 header words of an llm.c token file, or None for another file."""

    with path.open("rb") as handle:
        raw = handle.read(LLMC_HEADER_BYTES)
    if len(raw) < LLMC_HEADER_BYTES:
        return None
    words = struct.unpack("<256i", raw)
    return words if words[0] == LLMC_MAGIC else None


def load_token_file(path: pathlib.Path, raw_dtype: str = "uint16",
                    data_format: str = "auto") -> np.ndarray:
    """A token shard as a 1-D (memory-mapped where possible) array.

    `.npy` files load as arrays, `.txt`/`.text` files as their bytes; other
    files are llm.c shards when their header carries the llm.c magic (or
    data_format == "llmc", which requires it), else raw arrays of `raw_dtype`
    (data_format == "raw" skips the header check). An llm.c shard must have
    version 1, a positive token count and exactly header + 2 x count bytes
    (the format of rig/tokens.py:333-372).
    """

    path = pathlib.Path(path).expanduser().resolve()
    if not path.is_file():
        raise FileNotFoundError(f"token data not found: {path}")
    if path.suffix == ".npy":
        arr = np.load(path, mmap_mode="r", allow_pickle=False)
        if arr.ndim != 1:
            raise ValueError(f"{path} holds a {arr.ndim}-D array; token files are 1-D")
        return arr
    if path.suffix in (".txt", ".text"):
        return np.frombuffer(path.read_bytes(), dtype=np.uint8)
    header = None if data_format == "raw" else _llmc_header(path)
    if header is None and data_format == "llmc":
        raise ValueError(f"{path} lacks the llm.c header (magic {LLMC_MAGIC})")
    if header is not None:
        version, count = header[1], header[2]
        if version != LLMC_VERSION:
            raise ValueError(f"{path}: llm.c version {version} (only {LLMC_VERSION} is read)")
        if count < 1:
            raise ValueError(f"{path}: llm.c header declares {count} tokens")
        size = path.stat().st_size
        if size != LLMC_HEADER_BYTES + 2 * count:
            raise ValueError(f"{path}: {size} bytes on disk, but the llm.c header implies "
                             f"{LLMC_HEADER_BYTES + 2 * count}")
        return np.memmap(path, dtype="<u2", mode="r", offset=LLMC_HEADER_BYTES, shape=(count,))
    dtype = np.dtype(raw_dtype)
    if path.stat().st_size % dtype.itemsize:
        raise ValueError(f"{path}: size is not a whole number of {dtype.name} tokens")
    return np.memmap(path, dtype=dtype, mode="r")


def write_llmc_shard(path: pathlib.Path, tokens: np.ndarray) -> str:
    """Writes uint16 tokens as an llm.c shard; returns the file's SHA-256."""

    tokens = np.asarray(tokens)
    if tokens.size and (tokens.min() < 0 or tokens.max() > 0xFFFF):
        raise ValueError("llm.c shards hold uint16 token ids")
    header = struct.pack("<3i", LLMC_MAGIC, LLMC_VERSION, len(tokens)).ljust(LLMC_HEADER_BYTES,
                                                                             b"\0")
    path = pathlib.Path(path)
    with path.open("wb") as handle:
        handle.write(header)
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
