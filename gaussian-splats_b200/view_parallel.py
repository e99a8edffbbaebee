"""View-parallel rendering/training across GPUs (one process per GPU).

Every rank holds the whole scene, renders its own cameras forward and backward,
and the parameter gradients are summed with one all-reduce per step -- the
only exchange. The reference is single-device (training/train.py:125-151
renders one view per step); this is the multi-GPU shape of that step.

Gradients land in one flat float32 arena: before the backward each
parameter's ``.grad`` is made a view into the arena, so autograd accumulates
straight into it and the all-reduce runs on the arena with no packing.
"""

from __future__ import annotations

import datetime
import os
from collections.abc import Callable, Sequence

import torch
import torch.distributed as dist

PARAMETER_NAMES = ("mean", "rotation", "scale", "opacity", "color")


def shard_views(num_views: int, world_size: int, rank: int) -> list[int]:
    """Views of one rank: contiguous blocks, the first ``num_views % world``
    ranks taking one extra. Every view goes to exactly one rank."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside world of size {world_size}")
    base, extra = divmod(num_views, world_size)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (1 if rank < extra else 0)))


class GradientArena:
    """One flat buffer backing the ``.grad`` of a list of parameters."""

    def __init__(self, parameters: Sequence[torch.Tensor]):
        self.parameters = list(parameters)
        total = sum(p.numel() for p in self.parameters)
        device = self.parameters[0].device
        self.flat = torch.zeros(total, dtype=torch.float32, device=device)
        self.views = []
        offset = 0
        for p in self.parameters:
            self.views.append(self.flat[offset:offset + p.numel()].view_as(p))
            offset += p.numel()

    def attach(self) -> None:
        """Zero the arena and point every parameter's ``.grad`` into it."""
        self.flat.zero_()
        for p, v in zip(self.parameters, self.views):
            p.grad = v

    def check_attached(self) -> None:
        """Raise if autograd replaced a ``.grad`` instead of accumulating."""
        for p, v in zip(self.parameters, self.views):
            if p.grad is None or p.grad.data_ptr() != v.data_ptr():
                raise RuntimeError("a parameter gradient left the arena; call attach() "
                                   "before backward and do not reassign .grad")

    def all_reduce(self, group=None, average: bool = False) -> None:
        """Sum (or average) the arena over the process group."""
        self.check_attached()
        if dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)
            if average:
                self.flat.div_(dist.get_world_size(group))


def init_from_env(backend: str = "nccl", timeout_s: float = 120.0) -> tuple[int, int, int]:
    """Join the torchrun process group (RANK/WORLD_SIZE/MASTER_* from the
    environment) with a short collective timeout, so a rank that dies or never
    arrives ends the others' next collective with an error instead of a hang.
    Returns (rank, local_rank, world_size)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    return rank, local_rank, world


def train_step(
    splats,
    cameras: Sequence,
    targets: Sequence[torch.Tensor],
    arena: GradientArena,
    render: Callable,
    loss_fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor],
    group=None,
) -> torch.Tensor:
    """Forward + backward of this rank's views, then one all-reduce.

    ``render(splats, camera)`` returns an image; ``loss_fn(image, target)`` a
    scalar. Returns this rank's summed loss (a device tensor; no host sync).
    """
    arena.attach()
    total = None
    for camera, target in zip(cameras, targets):
        loss = loss_fn(render(splats, camera), target)
        loss.backward()
        total = loss.detach() if total is None else total + loss.detach()
    arena.all_reduce(group)
    return total if total is not None else torch.zeros((), device=arena.flat.device)
