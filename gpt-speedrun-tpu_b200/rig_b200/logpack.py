"""The `.riglog` container for a run's per-step scalars (docs/RIGLOG_FORMAT.md
of the rig; writer rig/logpack.py:59-300, reader :340-395).

Little-endian. An 8-byte magic, a 24-byte header (column count, 4 bytes of
padding, tokens per step, FLOPs per token), a table of 24-byte column entries
(metric id, scope id, layer, second index, element count), then fixed-width
records of one int32 step and one float32 per column. Columns are addressed by
permanent registry ids (rig/metrics.py), never by position or name, so a
reader of the rig opens these files unchanged.

Only the registry entries the training step writes are defined here; an
unknown name raises, as the rig's `column()` does.
"""

from __future__ import annotations

import dataclasses
import pathlib
import struct
from typing import BinaryIO, Iterable, Sequence

import numpy as np

MAGIC = b"RIGLOG\x00\x01"
SUFFIX = ".riglog"

# Permanent registry ids of rig/metrics.py (add-only upstream).
METRIC_IDS = {"step": 1, "tokens_processed": 2, "cumulative_flops": 3, "train_loss": 4,
              "learning_rate": 5, "grad_norm": 6, "router.balance_loss": 7,
              "router.max_load": 8, "router.min_load": 9, "router.load": 10,
              "router.entropy": 11, "router.top1_gate": 12, "router.logit_rms": 13}
# scope name -> (id, layered, indexed); "expert" is one routed expert of one block
SCOPE_IDS = {"overall": (1, False, False), "embeddings": (2, False, False),
             "unembedding": (3, False, False), "block": (4, True, False),
             "final_norm": (5, False, False), "expert": (6, True, True)}

_HEADER = struct.Struct("<i4xqd")          # column_count, pad, tokens_per_step, flops_per_token
_ENTRY = struct.Struct("<iiiiq")           # metric, scope, layer, index, element_count
assert _HEADER.size == 24 and _ENTRY.size == 24


@dataclasses.dataclass(frozen=True)
class Column:
    metric_id: int
    scope_id: int
    layer: int = -1
    index: int = -1
    element_count: int = 0


def column(metric_name: str, scope_name: str = "overall", layer: int | None = None,
           element_count: int = 0, index: int | None = None) -> Column:
    if metric_name not in METRIC_IDS:
        raise KeyError(f"unregistered metric {metric_name!r}")
    if scope_name not in SCOPE_IDS:
        raise KeyError(f"unregistered scope {scope_name!r}")
    scope_id, layered, indexed = SCOPE_IDS[scope_name]
    if layered and layer is None:
        raise ValueError(f"scope {scope_name!r} requires a layer index")
    if not layered and layer is not None:
        raise ValueError(f"scope {scope_name!r} does not take a layer index")
    if indexed and index is None:
        raise ValueError(f"scope {scope_name!r} requires a second index")
    if not indexed and index is not None:
        raise ValueError(f"scope {scope_name!r} does not take a second index")
    return Column(METRIC_IDS[metric_name], scope_id, -1 if layer is None else int(layer),
                  -1 if index is None else int(index), int(element_count))


class LogWriter:
    """Writes the header and column table on open, then one flushed record per
    `append`, so the file is a valid log after every append."""

    def __init__(self, path: pathlib.Path, columns: Sequence[Column], *, tokens_per_step: int,
                 flops_per_token: float):
        if not columns:
            raise ValueError("a log needs at least one column")
        if tokens_per_step <= 0 or flops_per_token <= 0:
            raise ValueError("tokens_per_step and flops_per_token must be positive")
        self.path = pathlib.Path(path)
        self.columns = tuple(columns)
        self._tokens = int(tokens_per_step)
        self._flops = float(flops_per_token)
        self._last = 0
        self._fh: BinaryIO | None = None

    def __enter__(self) -> "LogWriter":
        self._open()
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def _open(self) -> BinaryIO:
        if self._fh is None:
            self.path.parent.mkdir(parents=True, exist_ok=True)
            fh = self.path.open("wb")
            fh.write(MAGIC)
            fh.write(_HEADER.pack(len(self.columns), self._tokens, self._flops))
            for c in self.columns:
                fh.write(_ENTRY.pack(c.metric_id, c.scope_id, c.layer, c.index, c.element_count))
            fh.flush()
            self._fh = fh
        return self._fh

    def append(self, step: int, values: Iterable[float]) -> None:
        if step <= self._last:
            raise ValueError(f"log steps must increase; got {step} after {self._last}")
        row = np.asarray(list(values), dtype="<f4")
        if row.shape != (len(self.columns),):
            raise ValueError(f"expected {len(self.columns)} values, got {row.shape}")
        fh = self._open()
        fh.write(struct.pack("<i", int(step)) + row.tobytes())
        fh.flush()
        self._last = int(step)

    def close(self) -> None:
        if self._fh is not None:
            self._fh.close()
            self._fh = None


@dataclasses.dataclass(frozen=True)
class Log:
    columns: tuple[Column, ...]
    steps: np.ndarray
    values: np.ndarray
    tokens_per_step: int
    flops_per_token: float


def read_log(path: pathlib.Path) -> Log:
    """Reads a log; a partial trailing record is dropped."""

    raw = pathlib.Path(path).read_bytes()
    if not raw.startswith(MAGIC):
        raise ValueError(f"{path} is not a riglog file")
    n, tokens, flops = _HEADER.unpack_from(raw, len(MAGIC))
    off = len(MAGIC) + _HEADER.size
    cols = tuple(Column(*_ENTRY.unpack_from(raw, off + i * _ENTRY.size)) for i in range(n))
    off += n * _ENTRY.size
    rec = np.dtype([("step", "<i4"), ("values", "<f4", (n,))])
    count = (len(raw) - off) // rec.itemsize
    recs = np.frombuffer(raw, dtype=rec, count=count, offset=off)
    return Log(cols, recs["step"].copy(), recs["values"].copy(), int(tokens), float(flops))
