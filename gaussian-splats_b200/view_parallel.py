"""View-parallel rendering/training across GPUs (one process per GPU).

Every rank holds the whole scene, renders its own cameras forward and backward,
and the parameter gradients are summed with one all-reduce per step -- the
only exchange. The reference is single-device (training/train.py:125-151
renders one view per step); this is the multi-GPU shape of that step.

Gradients stay in the tensors autograd creates; the rasterizer's backward
returns them as views of one buffer, and the exchange is one all-reduce of
that buffer (no packing copy).
"""

from __future__ import annotations

import contextlib
import ctypes
import datetime
import os
from collections.abc import Callable, Sequence

import torch
import torch.distributed as dist

PARAMETER_NAMES = ("mean", "rotation", "scale", "opacity", "color")

# The group of the enclosing screen_space_exchange. Process-wide rather than
# thread-local: autograd runs CUDA backward functions on its own device
# thread, not on the thread that entered the context and called backward().
_EXCHANGE_GROUP = None


# Collectives this process has issued through this module; a CUDA-graph
# capture (gaussian_splats_b200.graphs) refuses steps that issue any.
COLLECTIVE_CALLS = 0


def _count_collective() -> None:
    global COLLECTIVE_CALLS
    COLLECTIVE_CALLS += 1


@contextlib.contextmanager
def screen_space_exchange(group=None):
    """Inside this context the rasterizer's backward returns the parameter
    gradients summed over every rank's view, computed without exchanging them.

    Each rank all-gathers the other ranks' screen-space gradients -- the 9
    floats per Gaussian that compositing backward produces -- with their tile
    counts and cameras, and runs one projection backward over all views
    (``gs_project_bwd_views``: parameters read once, each view's conic
    recomputed). That moves 40 bytes per Gaussian per rank instead of the 236
    bytes of parameter gradients an all-reduce moves at SH degree 3, for one
    extra pass of cheap per-view arithmetic.

    Preconditions: every rank runs the rasterizer's backward the same number
    of times inside the context (once per step in ``train_step``), and the
    loss reaches the Gaussian parameters only through rendered images (a
    regulariser on the parameters themselves would stay rank-local).
    """
    global _EXCHANGE_GROUP
    previous = _EXCHANGE_GROUP
    _EXCHANGE_GROUP = group if group is not None else dist.group.WORLD
    try:
        yield
    finally:
        _EXCHANGE_GROUP = previous


def active_exchange():
    """The process group of the enclosing :func:`screen_space_exchange`, or None."""
    group = _EXCHANGE_GROUP
    if group is None or not dist.is_initialized():
        return None
    return group


# Largest world size at which the screen-space exchange beats the all-reduce
# for one view per rank, per transport. Copying every rank's whole gradient
# (40 B per Gaussian from each peer) and summing all W views on every rank
# grows by ~55 us of arithmetic per extra view at 1M Gaussians, SH3, so past 4
# ranks the 236 MB all-reduce wins; the sharded form moves 40 B per Gaussian of
# its own shard from each peer plus the other shards' gradients and splits
# the arithmetic W ways, so it takes every world size the exchange supports.
SCREEN_EXCHANGE_MAX_WORLD = {"p2p": 4, "nccl": 4, "p2p-shard": 8, "auto": 8}


def screen_exchange_pays(world_size: int, transport: str | None = None) -> bool:
    """Whether ``train_step`` with one view per rank should use the
    screen-space exchange (over ``transport``, by default the module's) rather
    than the parameter-gradient all-reduce."""
    limit = SCREEN_EXCHANGE_MAX_WORLD[transport or EXCHANGE_TRANSPORT]
    return 1 < world_size <= limit


# How the screen-space exchange moves the gradients, all through symmetric
# memory peer-mapped over NVLink (one node, one GPU per rank) except "nccl":
# "p2p-shard" -- each rank copies its shard's rows of every rank's gradient,
#     computes the summed projection backward of its shard, and copies the
#     other ranks' finished shards (gs_exchange_gather_rows ..
#     gs_exchange_gather_shards);
# "p2p" -- each rank copies every rank's whole screen-space gradient and
#     computes the summed projection backward of all Gaussians;
# "nccl" -- three NCCL all-gathers, then as "p2p";
# "auto" -- "p2p" for two ranks, "p2p-shard" for more. On B200s with 1M
# Gaussians, SH3 (steps replayed from CUDA graphs): 2 ranks 1.88 ms per step
# whole vs 1.96 sharded (each rank has only one peer to copy 40 MB from, while
# the shard exchange copies 118 MB of parameter gradients); 4 ranks 2.29 ms
# whole vs 2.10 sharded.
EXCHANGE_TRANSPORT = "auto"
PEER_TRANSPORTS = ("p2p", "p2p-shard")


def transport_for(group=None) -> str:
    """The transport the screen-space exchange uses in ``group``."""
    if EXCHANGE_TRANSPORT != "auto":
        return EXCHANGE_TRANSPORT
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    return "p2p" if world <= 2 else "p2p-shard"


class PeerArena:
    """This rank's exchange arena in symmetric memory and every rank's arena
    as mapped here (``gs_peer_group``), for one Gaussian count.

    Holds the screen-space gradient [n, 9] that compositing backward writes,
    the tile counts [n], this rank's 29-word view record and the step flags
    of the peer handshake (see ``gs_exchange_publish``). Created once per
    (count, device, group) by all ranks together, outside graph capture."""

    def __init__(self, n: int, device: torch.device, group, num_sh: int | None = None):
        import torch.distributed._symmetric_memory as symm_mem

        from . import native

        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("the peer exchange arena is created by an eager step, not "
                               "inside graph capture")
        world = dist.get_world_size(group)
        if world > native.GS_MAX_PEERS:
            raise ValueError(f"the peer exchange takes at most {native.GS_MAX_PEERS} ranks")
        # one GPU per rank: the handshake kernels of two ranks must never share one
        gpus = [None] * world
        dist.all_gather_object(gpus, (os.uname().nodename, str(torch.cuda.get_device_properties(
            device).uuid)), group=group)
        if len(set(gpus)) != world or len({host for host, _ in gpus}) != 1:
            raise RuntimeError("the peer exchange needs one GPU per rank on one node")
        lib = native.lib()
        layout = native.ExchangeLayout()
        native.check(lib.gs_exchange_layout_for(n, world, ctypes.byref(layout)),
                     "gs_exchange_layout_for")
        # sharded: the arena also holds this rank's shard of parameter gradients
        self.sharded = num_sh is not None
        total = int(layout.bytes)
        if self.sharded:
            self.shard = native.ShardLayout()
            native.check(lib.gs_exchange_shard_layout(n, world, num_sh, ctypes.byref(self.shard)),
                         "gs_exchange_shard_layout")
            total = int(self.shard.bytes)
        buffer = symm_mem.empty(total, dtype=torch.uint8, device=device)
        buffer.zero_()
        torch.cuda.synchronize(device)
        handle = symm_mem.rendezvous(buffer, group)
        if handle.world_size != world:
            raise RuntimeError("symmetric memory group does not match the process group")
        offset = buffer.data_ptr() - handle.buffer_ptrs[handle.rank]
        if offset < 0 or offset + total > handle.buffer_size:
            raise RuntimeError("exchange arena lies outside its symmetric buffer")
        arenas = [int(base) + offset for base in handle.buffer_ptrs]
        if any(address % 256 for address in arenas):
            raise RuntimeError("exchange arenas must be 256-byte aligned")
        self.n, self.layout, self.buffer, self.handle = n, layout, buffer, handle
        slots = arenas + [None] * (native.GS_MAX_PEERS - world)
        self.group = native.PeerGroup(handle.rank, world,
                                      (ctypes.c_void_p * native.GS_MAX_PEERS)(*slots))
        self.grad_projected = buffer[layout.grad_projected:layout.grad_projected + 36 * n] \
            .view(torch.float32).view(n, 9)
        self.counts = buffer[layout.counts:layout.counts + 4 * n].view(torch.int32)
        self.record = buffer[layout.record:layout.record + 4 * native.VIEW_RECORD_WORDS] \
            .view(torch.int32)
        # the gradients and counts copied here each step: every rank's rows of
        # this rank's shard (sharded), or the peers' whole arrays
        rows = int(self.shard.rows) if self.sharded else n
        self.gathered_grad = torch.empty((world, rows, 9), dtype=torch.float32, device=device)
        self.gathered_counts = torch.empty((world, rows), dtype=torch.int32, device=device)


# Exchange arenas by (Gaussian count, device, id of the process group). Each
# entry holds its group object, so that id cannot be handed to another group
# while the entry lives: a group created after destroy_process_group() --
# even one with the same name, which torch reuses after a re-initialisation --
# is a different object and gets an arena of its own.
_ARENAS: dict = {}


def _resolve(group):
    return group if group is not None else dist.group.WORLD


def peer_arena(n: int, device: torch.device, group, num_sh: int | None = None) -> PeerArena:
    """The exchange arena for ``n`` Gaussians on ``device`` in ``group`` --
    sharded, with room for a shard of parameter gradients with ``num_sh`` SH
    coefficients, when ``num_sh`` is given -- created on first use, by every
    rank of the group in the same step."""
    group = _resolve(group)
    key = (n, num_sh, device.index, id(group))
    entry = _ARENAS.get(key)
    if entry is None or entry[0] is not group:
        entry = _ARENAS[key] = (group, PeerArena(n, device, group, num_sh))
    return entry[1]


def release_arenas(group=None) -> int:
    """Free this process's exchange arenas of ``group`` (of every group when
    None) and return how many were dropped. Call it before
    ``destroy_process_group``: an arena belongs to its group (its symmetric
    memory handle, peer mappings and step counters), and the group's ranks
    must not use it again. Every rank of the group calls it at the same point,
    with nothing of the exchange in flight."""
    doomed = [key for key, (owner, _) in _ARENAS.items()
              if group is None or owner is _resolve(group)]
    for key in doomed:
        del _ARENAS[key]
    return len(doomed)


def check_exchange() -> None:
    """Raise if any bounded wait of this rank's peer exchanges gave up (a
    peer that did not reach the same step within about a second).
    Synchronises the current stream."""
    from . import native

    for _, arena in _ARENAS.values():
        with torch.cuda.device(arena.buffer.device):
            stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            native.check(native.lib().gs_exchange_status(ctypes.byref(arena.group), stream),
                         "peer exchange (a rank did not reach the same step)")


def exchange_screen_gradients(grad_projected: torch.Tensor, counts: torch.Tensor,
                              record: torch.Tensor, group) -> tuple[torch.Tensor, ...]:
    """All-gather every rank's screen-space gradient [N, 9], tile counts [N]
    and 29-word view record; returns ([W, N, 9], [W, N], [W, 29]) on the
    gradients' device, in rank order."""
    _count_collective()
    world = dist.get_world_size(group)
    device = grad_projected.device
    n = grad_projected.shape[0]
    all_gp = grad_projected.new_empty((world, n, 9))
    all_counts = counts.new_empty((world, n))
    all_views = torch.empty((world, record.numel()), dtype=torch.int32, device=device)
    local_view = record.to(device).contiguous()
    # Three collectives, not one coalesced group: the tensors differ in dtype.
    works = [dist.all_gather_into_tensor(all_gp, grad_projected.contiguous(), group=group,
                                         async_op=True),
             dist.all_gather_into_tensor(all_counts, counts.contiguous(), group=group,
                                         async_op=True),
             dist.all_gather_into_tensor(all_views, local_view, group=group, async_op=True)]
    for work in works:
        work.wait()
    return all_gp, all_counts, all_views


def shard_views(num_views: int, world_size: int, rank: int) -> list[int]:
    """Views of one rank: contiguous blocks, the first ``num_views % world``
    ranks taking one extra. Every view goes to exactly one rank."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside world of size {world_size}")
    base, extra = divmod(num_views, world_size)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (1 if rank < extra else 0)))


def _shared_flat(grads: Sequence[torch.Tensor]) -> torch.Tensor | None:
    """One flat tensor over the storage the gradients share, if they are
    contiguous views that tile it exactly (as the rasterizer's backward returns
    them); else None."""
    storage = grads[0].untyped_storage()
    if any(g.untyped_storage().data_ptr() != storage.data_ptr() or not g.is_contiguous()
           or g.dtype != torch.float32 for g in grads):
        return None
    spans = sorted((g.storage_offset(), g.numel()) for g in grads)
    end = 0
    for offset, numel in spans:
        if offset != end:
            return None
        end += numel
    if end * 4 != storage.nbytes():
        return None
    return torch.empty(0, dtype=torch.float32, device=grads[0].device).set_(
        storage, 0, (end,), (1,))


def all_reduce_gradients(parameters: Sequence[torch.Tensor], group=None,
                         average: bool = False) -> None:
    """Sum (or average) every parameter's ``.grad`` over the process group.

    The gradients stay where autograd put them (no packing copy and no
    pre-zeroed buffer to accumulate into). When they are views of one buffer
    -- the rasterizer's backward returns them that way -- that buffer is
    all-reduced as one flat tensor: on B200s the 236 MB of a 1M-Gaussian SH3
    scene take 0.63 ms at 4 GPUs as one tensor, 0.75 ms as five and 0.82 ms
    coalesced. Otherwise each tensor is all-reduced on its own, back to back
    asynchronously. Parameters without a gradient on this rank take part with
    zeros so every rank issues the same collectives.
    """
    if not (dist.is_initialized() and dist.get_world_size(group) > 1):
        return
    _count_collective()
    grads = []
    for p in parameters:
        if p.grad is None:
            p.grad = torch.zeros_like(p)
        grads.append(p.grad)
    flat = _shared_flat(grads)
    if flat is not None:
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    else:
        works = [dist.all_reduce(g, op=dist.ReduceOp.SUM, group=group, async_op=True)
                 for g in grads]
        for work in works:
            work.wait()
    if average:
        size = dist.get_world_size(group)
        for p in parameters:
            p.grad.div_(size)


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
    parameters: Sequence[torch.Tensor],
    render: Callable,
    loss_fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor],
    group=None,
    screen_exchange: bool = False,
) -> torch.Tensor:
    """Forward + backward of this rank's views, then the gradient exchange.

    ``render(splats, camera)`` returns an image; ``loss_fn(image, target)`` a
    scalar. Gradients of ``parameters`` start from None, accumulate over this
    rank's views and are summed over ranks: by all-reducing them, or, with
    ``screen_exchange`` (one view per rank, image losses only; see
    :func:`screen_space_exchange`), inside the rasterizer's backward. Returns
    this rank's summed loss (a device tensor; no host sync).
    """
    for p in parameters:
        p.grad = None
    distributed = dist.is_initialized() and dist.get_world_size(group) > 1
    if screen_exchange and distributed and len(cameras) != 1:
        raise ValueError("screen_exchange needs exactly one view per rank and step")
    exchange = screen_space_exchange(group) if screen_exchange and distributed \
        else contextlib.nullcontext()
    total = None
    for camera, target in zip(cameras, targets):
        loss = loss_fn(render(splats, camera), target)
        with exchange:
            loss.backward()
        total = loss.detach() if total is None else total + loss.detach()
    if not (screen_exchange and distributed):
        all_reduce_gradients(parameters, group)
    if total is None:
        total = torch.zeros((), device=parameters[0].device)
    return total
