"""Data-parallel plumbing: one process per GPU, NCCL over NVLink.

Replaces rig/mesh.py (jax.distributed initialize :117-144, host-local batch
placement :179-190) and the XLA-inserted gradient all-reduce of the
reference's jitted step (recipes/reference/train.py:1773-1777: parameters and
optimizer state replicated, batch sharded over the "data" axis).

The global batch is split contiguously by rank exactly like
rig/tokens.py:256-260. The loss cotangent already carries 1/(tokens * world),
so a SUM all-reduce of the gradients gives the gradient of the global mean
loss. `GradientReducer` launches one asynchronous all-reduce per transformer
block as soon as that block's backward kernels are enqueued (NCCL waits on the
compute stream at launch, then runs concurrently with the rest of the
backward), plus one for the embedding/final-norm tail; `finish` makes the
compute stream wait for all of them before the optimizer runs.
"""

from __future__ import annotations

import datetime
import math
import os

import torch
import torch.distributed as dist


def initialize_distributed_runtime(backend: str = "nccl", timeout_s: float = 600.0):
    """Initializes torch.distributed from torchrun's environment variables.

    Returns (rank, world_size, local_rank). A single process without the
    environment runs with world_size 1 and no process group.
    """

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(
            backend=backend,
            rank=rank,
            world_size=world,
            timeout=datetime.timedelta(seconds=timeout_s),
            device_id=torch.device("cuda", local) if backend == "nccl" else None,
        )
    return rank, world, local


def local_batch_slice(global_batch: int, rank: int, world: int) -> slice:
    """Rows of the global batch owned by `rank` (rig/tokens.py:256-260)."""

    if global_batch % world:
        raise ValueError("global batch size must be divisible by process count")
    local = global_batch // world
    return slice(rank * local, (rank + 1) * local)


class GradientReducer:
    """Bucketed, backward-overlapped SUM all-reduce over a flat gradient buffer."""

    def __init__(self, grads: torch.Tensor, group=None, on_reduced=None):
        self.grads = grads
        self.group = group
        self.works = []
        # on_reduced(start, end, work): called right after a bucket's
        # all-reduce is launched, e.g. to queue its optimizer update behind it
        self.on_reduced = on_reduced

    def launch(self, start: int, end: int) -> None:
        work = dist.all_reduce(self.grads[start:end], op=dist.ReduceOp.SUM, group=self.group,
                               async_op=True)
        self.works.append(work)
        if self.on_reduced is not None:
            self.on_reduced(start, end, work)

    def finish(self, loss: torch.Tensor | None = None) -> None:
        """Waits for every bucket; `loss` (this rank's mean) becomes the global mean."""

        if loss is not None:
            self.works.append(
                dist.all_reduce(loss, op=dist.ReduceOp.SUM, group=self.group, async_op=True))
        for w in self.works:
            w.wait()
        self.works.clear()
        if loss is not None:
            loss.div_(dist.get_world_size(self.group))


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier()


def finite_metric(name: str, value: float, *, positive: bool = False) -> float:
    """A host-side metric checked before it is logged (rig/mesh.py:214-223):
    NaN, infinities, negatives, and zero when `positive`, raise
    FloatingPointError, which ends the run the way the reference's does."""

    value = float(value)
    low_ok = value > 0.0 if positive else value >= 0.0
    if math.isfinite(value) and low_ok:
        return value
    need = "finite and positive" if positive else "finite and nonnegative"
    raise FloatingPointError(f"{name} must be {need}, got {value!r}")
