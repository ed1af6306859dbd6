"""Data-parallel host logic on CPU with the gloo backend (world size 2):
bucketed, overlapped gradient all-reduce and the rank split of the batch."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rig_b200.mesh import GradientReducer, local_batch_slice


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        grads = torch.arange(100, dtype=torch.float32) * (rank + 1)
        loss = torch.tensor([float(rank + 1)])
        red = GradientReducer(grads)
        # blocks finish in reverse order during backward; the tail goes last
        for start, end in ((60, 100), (20, 60), (0, 20)):
            red.launch(start, end)
        red.finish(loss)
        out[rank] = (grads.numpy().copy(), float(loss.item()))
    finally:
        dist.destroy_process_group()


def _worker_with_updates(rank, world, port, out):
    """Each bucket's update is queued right behind its all-reduce (on_reduced)
    and, after waiting on that work, sees the summed gradient of its range."""

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        grads = torch.arange(100, dtype=torch.float32) * (rank + 1)
        params = torch.zeros(100)
        seen = []

        def update(start, end, work):
            work.wait()
            params[start:end] -= 0.5 * grads[start:end]
            seen.append((start, end))

        red = GradientReducer(grads, on_reduced=update)
        for start, end in ((60, 100), (20, 60), (0, 20)):
            red.launch(start, end)
        red.finish(torch.tensor([1.0]))
        out[rank] = (params.numpy().copy(), seen)
    finally:
        dist.destroy_process_group()


def test_gradient_reducer_bucket_updates_gloo():
    world = 2
    port = _free_port()
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_worker_with_updates, args=(world, port, out), nprocs=world, join=True)
    for r in range(world):
        params, seen = out[r]
        np.testing.assert_array_equal(params, -0.5 * 3.0 * np.arange(100, dtype=np.float32))
        assert seen == [(60, 100), (20, 60), (0, 20)]


def test_gradient_reducer_gloo():
    world = 2
    port = _free_port()
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
    expect = np.arange(100, dtype=np.float32) * 3.0  # rank 0 x1 + rank 1 x2
    for r in range(world):
        g, loss = out[r]
        np.testing.assert_array_equal(g, expect)
        assert loss == pytest.approx(1.5)


def test_local_batch_slices_partition_the_global_batch():
    rows = [local_batch_slice(128, r, 8) for r in range(8)]
    assert [s.start for s in rows] == list(range(0, 128, 16))
    assert all(s.stop - s.start == 16 for s in rows)
    with pytest.raises(ValueError):
        local_batch_slice(128, 0, 3)


def test_finite_metric_raises_like_the_reference():
    import math

    import pytest

    from rig_b200.mesh import finite_metric

    assert finite_metric("loss", 2.5) == 2.5
    assert finite_metric("lr", 0.0) == 0.0
    for bad in (math.nan, math.inf, -1.0):
        with pytest.raises(FloatingPointError):
            finite_metric("loss", bad)
    with pytest.raises(FloatingPointError):
        finite_metric("tokens_per_second", 0.0, positive=True)


def test_tail_parts_cover_the_bucket():
    """The tail bucket is reduced and updated in contiguous parts that tile it
    exactly, with inner boundaries 1024-element aligned (the AdamW range entry
    point needs multiples of 4)."""

    from rig_b200.config import load_config
    from rig_b200.model import ParamLayout, tail_parts

    layout = ParamLayout(load_config("baseline_125m"))
    start, end = layout.tail_range
    parts = tail_parts(start, end)
    assert len(parts) == 4 and parts[0][0] == start and parts[-1][1] == end
    assert all(a < b for a, b in parts)
    assert all(parts[i][1] == parts[i + 1][0] for i in range(len(parts) - 1))
    assert all((b - start) % 1024 == 0 for _, b in parts[:-1]) and start % 4 == 0
    assert tail_parts(100, 200) == [(100, 200)]
