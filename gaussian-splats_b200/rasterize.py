"""The ``gaussian_splats::rasterize`` operator on the B200 kernels.

Same operator name, 19-argument schema, 10 outputs and autograd contract as
the reference's Triton operator (kernels/rasterize/interface.py:17-244), so
code written against ``torch.ops.gaussian_splats.rasterize`` or against the
``rasterize(splats, camera, ...)`` helpers runs unchanged. (Registering the
same operator name as the reference means the two cannot be imported into one
process.)

The stages run as hand-written sm_100a kernels through the C ABI of
``libgs_b200.so`` (``include/gs_b200.h``), on the current CUDA stream:

1. ``gs_project_fwd``   projection, SH colour, opacity, tile rectangle and count,
                        and each Gaussian's 64-byte record for the compositors;
2. ``gs_bin_count``     depth order of the visible Gaussians and the
                        intersection total -- the one host sync, as in
                        intersections.py:51;
3. ``gs_bin_sort``      (tile, depth)-ordered Gaussian ids and tile ranges;
4. ``gs_composite_fwd`` per-tile front-to-back compositing.
Backward: ``gs_composite_bwd`` (on the forward's records, or on records
rebuilt by ``gs_pack_records``), then ``gs_project_bwd`` (interface.py:176-239).

Differences from the reference, all deliberate:
* ``ranges`` is int64 in the fake (meta) kernel too, matching what the real
  operator returns (the reference's fake declares int32, interface.py:146-153);
* an unknown ``rendering_mode`` raises ``ValueError`` instead of mixing the
  ellipsoid projection with Gaussian compositing;
* the backward covers SH degree 4 (coefficients 16..24 and their share of the
  view-direction gradient), which the reference leaves uninitialised
  (project_bwd.py:33,355), and ellipsoid rendering, which it refuses
  (interface.py:184-186);
* inputs must be CUDA tensors: there is no CPU path.
"""

from __future__ import annotations

import ctypes
import math
import os
from typing import Literal

import torch
from torch.utils.weak import WeakIdKeyDictionary

from . import native, view_parallel
from .camera import Camera

_OUTPUTS = 10
_VALID_MODES = ("gaussian", "ellipsoid")


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None and t.numel() else 0)


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _tile_order(ranges: torch.Tensor, n_contributors: torch.Tensor | None, pref,
                stream: ctypes.c_void_p) -> torch.Tensor:
    """The compositors' heavy-first visiting order of the view's tiles
    (gs_tile_order): by list length for the forward, by largest contributor
    count (``n_contributors`` given) for the backward."""
    num_tiles = ranges.shape[0]
    order = torch.empty((num_tiles,), dtype=torch.int32, device=ranges.device)
    work = torch.empty((num_tiles + 128,), dtype=torch.int32, device=ranges.device)
    native.check(native.lib().gs_tile_order(_ptr(ranges), _ptr(n_contributors), pref,
                                            _ptr(order), _ptr(work), stream), "gs_tile_order")
    return order


def _backward_plan(ranges: torch.Tensor, n_contributors: torch.Tensor, pref,
                   stream: ctypes.c_void_p) -> torch.Tensor:
    """The compositing backward's plan of the render (gs_composite_bwd_plan):
    tiles heaviest first, the longest walks split into parts."""
    lib = native.lib()
    plan = torch.empty((lib.gs_composite_bwd_plan_size(pref),), dtype=torch.uint8,
                       device=ranges.device)
    native.check(lib.gs_composite_bwd_plan(_ptr(ranges), _ptr(n_contributors), pref, 0,
                                           _ptr(plan), plan.numel(), stream),
                 "gs_composite_bwd_plan")
    return plan


def _check_inputs(mean: torch.Tensor, color: torch.Tensor, rendering_mode: str) -> None:
    if not mean.is_cuda:
        raise RuntimeError(
            "gaussian_splats_b200 runs on CUDA devices only (there is no CPU fallback); "
            f"got tensors on {mean.device}"
        )
    if color.shape[1] > 25:
        raise NotImplementedError(
            f"SH degrees above 4 are not implemented. Got {color.shape[1]}."
        )
    if rendering_mode not in _VALID_MODES:
        raise ValueError(f"Invalid rendering mode: {rendering_mode}")


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(torch.float32).contiguous()


# Device copies of host camera tensors: host tensor -> (its version, device,
# copy). Entries die with the host tensor.
_DEVICE_COPIES = WeakIdKeyDictionary()


def _to_device(t: torch.Tensor, device: torch.device) -> torch.Tensor:
    """``t`` on ``device``. A host tensor goes up through pinned memory with a
    non-blocking copy: a plain ``.to`` from pageable memory synchronises the
    stream, so the host would wait for all queued GPU work on every render and
    the GPU would then idle while the next kernels are launched. The copy is
    kept while the host tensor is unchanged (same object and version), so
    re-rendering a camera copies nothing."""
    if t.device == device or device.type != "cuda" or t.requires_grad:
        return t.to(device)
    cached = _DEVICE_COPIES.get(t)
    if cached is not None and cached[0] == t._version and cached[1] == device:
        return cached[2]
    if torch.cuda.is_current_stream_capturing():
        # a captured copy would read the staging buffer again on every replay
        raise RuntimeError("a host camera tensor changed during CUDA-graph capture; keep the "
                           "camera on the device, or render it once before capturing")
    staged = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    staged.copy_(t)
    copy = staged.to(device, non_blocking=True)
    _DEVICE_COPIES[t] = (t._version, device, copy)
    return copy


class StageTimer:
    """Records a CUDA event on the launching stream after each stage.

    Install with ``with StageTimer() as timer:``; ``timer.durations()`` then
    returns milliseconds per stage name summed over the recorded calls. Off
    (no events) unless installed.
    """

    active: "StageTimer | None" = None

    def __init__(self):
        self.marks: list[tuple[str, torch.cuda.Event]] = []

    def __enter__(self):
        StageTimer.active = self
        return self

    def __exit__(self, *exc):
        StageTimer.active = None

    def mark(self, name: str) -> None:
        event = torch.cuda.Event(enable_timing=True)
        event.record()
        self.marks.append((name, event))

    def durations(self) -> dict[str, float]:
        """Mean milliseconds between each ``begin:X`` mark and the ``X`` mark
        that follows it."""
        torch.cuda.synchronize()
        out: dict[str, float] = {}
        counts: dict[str, int] = {}
        for (first, before), (name, after) in zip(self.marks, self.marks[1:]):
            if first != "begin:" + name:
                continue
            out[name] = out.get(name, 0.0) + before.elapsed_time(after)
            counts[name] = counts.get(name, 0) + 1
        return {k: v / counts[k] for k, v in out.items()}


def _mark(name: str) -> None:
    if StageTimer.active is not None:
        StageTimer.active.mark(name)


# Intersection total of the last render per (Gaussians, tiles, device): later
# renders size their sort buffers from it (plus headroom) and enqueue the sort
# before their own total reaches the host.
_LAST_TOTAL: dict[tuple[int, int, int | None], int] = {}

# The graph capture in progress (gaussian_splats_b200.graphs sets it while a
# captured step runs), or None; and, while a step is warmed up for capture, the
# largest intersection total seen per key.
_CAPTURE = None
_SEEN_TOTALS: dict | None = None


# Records of renders whose backward has not run yet, by (counts storage
# address, Gaussian count): the operator's saved set is the reference's, so
# the forward's records ride along here instead. The address identifies the
# render: its counts tensor is saved for the backward, so no later render can
# reuse that storage while the backward is still to come. A backward that
# finds no entry (a second backward, or one beyond the last few renders)
# rebuilds the records from the saved outputs (gs_pack_records).
_PENDING_RECORDS: dict = {}
_MAX_PENDING_RECORDS = 4


def deterministic_backward() -> bool:
    """Whether the backward uses its order-fixed form (the same gradient bits
    on every run): with ``GAUSSIAN_SPLATS_B200_DETERMINISTIC=1`` in the
    environment, or under ``torch.use_deterministic_algorithms(True)``. The
    default adds each tile's contributions with float atomics, whose order
    varies from run to run in the last bits (the reference selects between its
    two forms with GAUSSIAN_SPLATS_ATOMIC_BACKWARD, interface.py:218)."""
    return (os.environ.get("GAUSSIAN_SPLATS_B200_DETERMINISTIC") == "1"
            or torch.are_deterministic_algorithms_enabled())


def _keep_records(counts: torch.Tensor, records: torch.Tensor) -> None:
    key = (counts.data_ptr(), counts.numel())
    _PENDING_RECORDS.pop(key, None)
    _PENDING_RECORDS[key] = records
    while len(_PENDING_RECORDS) > _MAX_PENDING_RECORDS:
        _PENDING_RECORDS.pop(next(iter(_PENDING_RECORDS)))


def _pinned_words() -> torch.Tensor:
    """Two zeroed pinned int64 host words (intersection total, error word) for
    one render; torch's pinned-memory cache makes them cheap to allocate."""
    return torch.zeros(2, dtype=torch.int64, pin_memory=True)


@torch.library.custom_op("gaussian_splats::rasterize", mutates_args=())
def _rasterize(
    mean: torch.Tensor,
    rotation: torch.Tensor,
    scale: torch.Tensor,
    opacity: torch.Tensor,
    color: torch.Tensor,
    camera_rotation: torch.Tensor,
    camera_translation: torch.Tensor,
    fx: float,
    fy: float,
    cx: float,
    cy: float,
    image_width: int,
    image_height: int,
    tile_size: int,
    opacity_threshold: float,
    near: float,
    far: float,
    rendering_mode: str,
    confidence: float,
) -> tuple[
    torch.Tensor,  # image [H, W, 3]
    torch.Tensor,  # final_transmittance [H, W]
    torch.Tensor,  # n_contributors [H, W] int32
    torch.Tensor,  # projected_mean [N, 3] (pixel x, pixel y, depth)
    torch.Tensor,  # inverse_covariance [N, 2, 2]
    torch.Tensor,  # projected_color [N, 3]
    torch.Tensor,  # projected_opacity [N, 1]
    torch.Tensor,  # gaussian_ids [I] int32
    torch.Tensor,  # ranges [tiles, 2] int64
    torch.Tensor,  # counts [N] int32
]:
    _check_inputs(mean, color, rendering_mode)
    lib = native.lib()
    device = mean.device
    backward_possible = any(t.requires_grad for t in (mean, rotation, scale, opacity, color))
    mean, rotation, scale, opacity, color = map(_f32, (mean, rotation, scale, opacity, color))
    camera_rotation, camera_translation = _f32(camera_rotation), _f32(camera_translation)
    n, num_sh = mean.shape[0], color.shape[1]
    params = native.make_params(fx, fy, cx, cy, image_width, image_height, tile_size,
                                opacity_threshold, near, far, rendering_mode, confidence)
    pref = ctypes.byref(params)
    num_tiles = (image_width // tile_size) * (image_height // tile_size)
    with torch.cuda.device(device):
        stream = _stream(device)
        projected_mean = mean.new_empty((n, 3))
        inverse_covariance = mean.new_empty((n, 2, 2))
        projected_color = mean.new_empty((n, 3))
        projected_opacity = mean.new_empty((n, 1))
        bounds = torch.empty((n, 4), dtype=torch.int32, device=device)
        counts = torch.empty((n,), dtype=torch.int32, device=device)
        records = mean.new_empty((n, 16))  # the compositors' staged form, internal
        _mark("begin:project_fwd")
        native.check(lib.gs_project_fwd(
            n, num_sh, _ptr(mean), _ptr(rotation), _ptr(scale), _ptr(opacity), _ptr(color),
            _ptr(camera_rotation), _ptr(camera_translation), pref, _ptr(projected_mean),
            _ptr(inverse_covariance), _ptr(projected_color), _ptr(projected_opacity),
            _ptr(bounds), _ptr(counts), _ptr(records), stream), "gs_project_fwd")
        _mark("project_fwd")

        count_bytes = lib.gs_bin_count_workspace_size(n)
        count_ws = torch.empty((count_bytes,), dtype=torch.uint8, device=device)
        ranges = torch.empty((num_tiles, 2), dtype=torch.int64, device=device)
        image = mean.new_empty((image_height, image_width, 3))
        final_transmittance = mean.new_empty((image_height, image_width))
        n_contributors = torch.empty((image_height, image_width), dtype=torch.int32,
                                     device=device)

        def sort_and_composite(capacity):
            gaussian_ids = torch.empty((capacity,), dtype=torch.int32, device=device)
            sort_bytes = lib.gs_bin_sort_workspace_size(n, capacity, pref)
            sort_ws = torch.empty((sort_bytes,), dtype=torch.uint8, device=device)
            _mark("begin:bin_sort")
            native.check(lib.gs_bin_sort(
                n, capacity, _ptr(bounds), _ptr(counts), pref, _ptr(count_ws), count_bytes,
                _ptr(sort_ws), sort_bytes, _ptr(gaussian_ids), _ptr(ranges), stream),
                "gs_bin_sort")
            _mark("bin_sort")
            if os.environ.get("GAUSSIAN_SPLATS_B200_CHECK") == "1" and \
                    not torch.cuda.is_current_stream_capturing():
                native.check(lib.gs_bin_check(_ptr(count_ws), _ptr(sort_ws), stream), "binning")
            _mark("begin:composite_fwd")
            order = _tile_order(ranges, None, pref, stream)
            native.check(lib.gs_composite_fwd(
                _ptr(records), _ptr(gaussian_ids), _ptr(ranges), pref, _ptr(image),
                _ptr(final_transmittance), _ptr(n_contributors), _ptr(order), stream),
                "gs_composite_fwd")
            _mark("composite_fwd")
            return gaussian_ids

        key = (n, num_tiles, device.index)
        last = _LAST_TOTAL.get(key)
        capture = _CAPTURE if torch.cuda.is_current_stream_capturing() else None
        _mark("begin:bin_count")
        if capture is not None:
            # Inside CUDA-graph capture: no host wait. The sort and compositing
            # run at the capture's capacity; a captured copy refreshes the
            # total and error words on every replay, and the graph's owner
            # checks them after each replay (gaussian_splats_b200.graphs).
            if last is None:
                raise RuntimeError("render each view once outside graph capture first: the "
                                   "first render sizes its intersection buffer")
            capacity = capture.capacity(key, last)
            words = capture.take_words()
            native.check(lib.gs_bin_count_async(
                n, _ptr(projected_mean), _ptr(counts), _ptr(count_ws), count_bytes,
                ctypes.c_void_p(words.data_ptr()), ctypes.c_void_p(words.data_ptr() + 8),
                stream), "gs_bin_count_async")
            _mark("bin_count")
            gaussian_ids = sort_and_composite(capacity)
            capture.record(key, capacity, words)
            total = None
        elif last is None:
            # First render of this shape: wait for the total, size exactly.
            total = ctypes.c_int64(0)
            native.check(lib.gs_bin_count(
                n, _ptr(projected_mean), _ptr(counts), _ptr(count_ws), count_bytes,
                ctypes.byref(total), stream), "gs_bin_count")
            total = total.value
            _mark("bin_count")
            gaussian_ids = sort_and_composite(total)
        else:
            # Enqueue the sort and compositing at a capacity sized from the
            # last total, read this total when the count phase is done (the
            # GPU keeps working meanwhile), and redo if it did not fit.
            words = _pinned_words()
            native.check(lib.gs_bin_count_async(
                n, _ptr(projected_mean), _ptr(counts), _ptr(count_ws), count_bytes,
                ctypes.c_void_p(words.data_ptr()), ctypes.c_void_p(words.data_ptr() + 8),
                stream), "gs_bin_count_async")
            counted = torch.cuda.Event()
            counted.record(torch.cuda.current_stream(device))
            _mark("bin_count")
            capacity = last + last // 4 + 4096
            gaussian_ids = sort_and_composite(capacity)
            counted.synchronize()
            total, error = int(words[0]), int(words[1]) & 0xFFFFFFFF
            if error:
                native.check(-6, "gs_bin_count_async")
            if total >= 1 << 30:
                native.check(-3, "gs_bin_count_async")
            if total > capacity:
                gaussian_ids = sort_and_composite(total)
            else:
                gaussian_ids.resize_(total)  # same storage, no copy
        if total is not None:
            _LAST_TOTAL[key] = total
            if _SEEN_TOTALS is not None:
                _SEEN_TOTALS[key] = max(total, _SEEN_TOTALS.get(key, 0))
        if backward_possible:
            _keep_records(counts, records)
    return (image, final_transmittance, n_contributors, projected_mean, inverse_covariance,
            projected_color, projected_opacity, gaussian_ids, ranges, counts)


@_rasterize.register_fake
def _rasterize_fake(mean, rotation, scale, opacity, color, camera_rotation, camera_translation,
                    fx, fy, cx, cy, image_width, image_height, tile_size, opacity_threshold,
                    near, far, rendering_mode, confidence):
    dynamic = torch.library.get_ctx().new_dynamic_size()
    n = mean.shape[0]
    num_tiles = (image_height // tile_size) * (image_width // tile_size)
    i32 = dict(dtype=torch.int32, device=mean.device)
    return (
        mean.new_empty((image_height, image_width, 3)),
        mean.new_empty((image_height, image_width)),
        torch.empty((image_height, image_width), **i32),
        mean.new_empty((n, 3)),
        mean.new_empty((n, 2, 2)),
        mean.new_empty((n, 3)),
        mean.new_empty((n, 1)),
        torch.empty((dynamic,), **i32),
        torch.empty((num_tiles, 2), dtype=torch.int64, device=mean.device),
        torch.empty((n,), **i32),
    )


def _setup_context(ctx, inputs, output) -> None:
    # Same saved set as interface.py:158-173: the 7 tensor inputs and outputs[1:].
    ctx.save_for_backward(*inputs[:7], *output[1:])
    # Only the image's gradient is used; do not materialise zero gradients for
    # the nine other outputs (one fill kernel each).
    ctx.set_materialize_grads(False)
    (ctx.fx, ctx.fy, ctx.cx, ctx.cy, ctx.image_width, ctx.image_height, ctx.tile_size,
     ctx.opacity_threshold, ctx.near, ctx.far, ctx.rendering_mode, ctx.confidence) = inputs[7:]


def _carve(flat: torch.Tensor, n: int, shapes) -> list[torch.Tensor]:
    """Consecutive views [n, *shape] of a flat buffer."""
    views, offset = [], 0
    for shape in shapes:
        size = n * math.prod(shape)
        views.append(flat[offset:offset + size].view(n, *shape))
        offset += size
    return views


def _backward(ctx, *grad_outputs):
    """Composite backward, then projection backward (interface.py:176-239).

    Unlike the reference (interface.py:184-186), ellipsoid rendering has a
    backward too: its indicator falloff passes gradients to colour and
    opacity only."""
    (mean, rotation, scale, opacity, color, camera_rotation, camera_translation,
     final_transmittance, n_contributors, projected_mean, inverse_covariance, projected_color,
     projected_opacity, gaussian_ids, ranges, counts) = ctx.saved_tensors
    lib = native.lib()
    device = mean.device
    grad_image = grad_outputs[0]
    if grad_image is None:
        grad_image = torch.zeros((ctx.image_height, ctx.image_width, 3), device=device)
    grad_image = _f32(grad_image)
    mean, rotation, scale, opacity, color = map(_f32, (mean, rotation, scale, opacity, color))
    camera_rotation, camera_translation = _f32(camera_rotation), _f32(camera_translation)
    n, num_sh = mean.shape[0], color.shape[1]
    params = native.make_params(ctx.fx, ctx.fy, ctx.cx, ctx.cy, ctx.image_width,
                                ctx.image_height, ctx.tile_size, ctx.opacity_threshold,
                                ctx.near, ctx.far, ctx.rendering_mode, ctx.confidence)
    pref = ctypes.byref(params)
    group = view_parallel.active_exchange()
    transport = view_parallel.transport_for(group) if group is not None else None
    peers = group is not None and transport in view_parallel.PEER_TRANSPORTS
    sharded = peers and transport == "p2p-shard"
    with torch.cuda.device(device):
        stream = _stream(device)
        if peers:
            # Peer exchange: the screen-space gradient goes straight into
            # this rank's arena, once every peer has finished reading it.
            arena = view_parallel.peer_arena(n, device, group, num_sh if sharded else None)
            group_ref = ctypes.byref(arena.group)
            _mark("begin:exchange_wait")
            native.check(lib.gs_exchange_begin(group_ref, stream), "gs_exchange_begin")
            _mark("exchange_wait")
            grad_projected = arena.grad_projected
        else:
            grad_projected = mean.new_empty((n, 9))
        # The compositors' records of this render: kept by its forward, or
        # rebuilt from the saved projection outputs.
        records = _PENDING_RECORDS.pop((counts.data_ptr(), counts.numel()), None)
        _mark("begin:composite_bwd")
        if records is None:
            records = mean.new_empty((n, 16))
            native.check(lib.gs_pack_records(
                n, _ptr(projected_mean), _ptr(inverse_covariance), _ptr(projected_color),
                _ptr(projected_opacity), pref, _ptr(records), stream), "gs_pack_records")
        if deterministic_backward():
            # order-fixed form: the same gradient bits on every run
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("the deterministic backward runs eagerly (a captured render's "
                                   "gaussian_ids is longer than its intersection total)")
            total = gaussian_ids.numel()
            order = _tile_order(ranges, n_contributors, pref, stream)
            ws_bytes = lib.gs_composite_bwd_deterministic_workspace_size(n, total)
            workspace = torch.empty((ws_bytes,), dtype=torch.uint8, device=device)
            native.check(lib.gs_composite_bwd_deterministic(
                n, total, _ptr(records), _ptr(gaussian_ids), _ptr(ranges), _ptr(grad_image),
                _ptr(final_transmittance), _ptr(n_contributors), pref, _ptr(workspace),
                ws_bytes, _ptr(grad_projected), _ptr(order), stream),
                "gs_composite_bwd_deterministic")
        else:
            plan = _backward_plan(ranges, n_contributors, pref, stream)
            native.check(lib.gs_composite_bwd(
                n, _ptr(records), _ptr(gaussian_ids), _ptr(ranges), _ptr(grad_image),
                _ptr(final_transmittance), _ptr(n_contributors), pref, _ptr(grad_projected),
                _ptr(plan), stream), "gs_composite_bwd")
        _mark("composite_bwd")
        # The five gradients are carved out of one buffer (rotation and colour
        # first, keeping their 16-byte rows aligned), so a view-parallel step
        # can all-reduce them as one flat tensor without a packing copy.
        grad_rotation, grad_color, grad_mean, grad_scale, grad_opacity = _carve(
            mean.new_empty((n * (11 + 3 * num_sh),)), n,
            ((4,), (num_sh, 3), (3,), (3,), (1,)))
        if group is not None:
            # View-parallel step: every rank's screen-space gradient and
            # camera, and the projection backward summed over all views.
            capture = _CAPTURE if torch.cuda.is_current_stream_capturing() else None
            record = native.view_record(params, camera_rotation, camera_translation,
                                        keep=capture.keep if capture is not None else None)
        if peers:
            arena.counts.copy_(counts)
            arena.record.copy_(record)
            _mark("begin:exchange_publish")
            native.check(lib.gs_exchange_publish(group_ref, n, stream), "gs_exchange_publish")
            _mark("exchange_publish")
        if sharded:
            # this rank's rows of every rank's gradient, the summed backward of
            # this rank's shard, then every rank's finished shard
            _mark("begin:exchange_rows")
            native.check(lib.gs_exchange_gather_rows(group_ref, n, _ptr(arena.gathered_grad),
                                                     _ptr(arena.gathered_counts), stream),
                         "gs_exchange_gather_rows")
            _mark("exchange_rows")
            _mark("begin:project_bwd")
            native.check(lib.gs_project_bwd_shard(
                n, num_sh, group_ref, _ptr(arena.gathered_grad), _ptr(arena.gathered_counts),
                _ptr(mean), _ptr(rotation), _ptr(scale), _ptr(opacity), _ptr(color), stream),
                "gs_project_bwd_shard")
            _mark("project_bwd")
            _mark("begin:exchange_shard_wait")
            native.check(lib.gs_exchange_publish_shard(group_ref, stream),
                         "gs_exchange_publish_shard")
            _mark("exchange_shard_wait")
            _mark("begin:exchange_shards")
            native.check(lib.gs_exchange_gather_shards(
                group_ref, n, num_sh, _ptr(grad_rotation), _ptr(grad_color), _ptr(grad_mean),
                _ptr(grad_scale), _ptr(grad_opacity), stream), "gs_exchange_gather_shards")
            _mark("exchange_shards")
            native.check(lib.gs_exchange_finish(group_ref, stream), "gs_exchange_finish")
        elif peers:
            # bulk copies of the peers' gradients over NVLink; the peers may
            # overwrite theirs as soon as the copies are done
            _mark("begin:exchange_rows")
            native.check(lib.gs_exchange_gather(group_ref, n, _ptr(arena.gathered_grad),
                                                _ptr(arena.gathered_counts), stream),
                         "gs_exchange_gather")
            _mark("exchange_rows")
            native.check(lib.gs_exchange_finish(group_ref, stream), "gs_exchange_finish")
            _mark("begin:project_bwd")
            native.check(lib.gs_project_bwd_peers(
                n, num_sh, group_ref, _ptr(arena.gathered_grad), _ptr(arena.gathered_counts),
                _ptr(mean), _ptr(rotation), _ptr(scale), _ptr(opacity), _ptr(color),
                _ptr(grad_mean), _ptr(grad_rotation), _ptr(grad_scale), _ptr(grad_opacity),
                _ptr(grad_color), stream), "gs_project_bwd_peers")
            _mark("project_bwd")
        elif group is not None:
            all_gp, all_counts, all_views = view_parallel.exchange_screen_gradients(
                grad_projected, counts, record, group)
            _mark("begin:project_bwd")
            native.check(lib.gs_project_bwd_views(
                n, num_sh, all_views.shape[0], _ptr(mean), _ptr(rotation), _ptr(scale),
                _ptr(opacity), _ptr(color), _ptr(all_views), _ptr(all_gp), _ptr(all_counts),
                _ptr(grad_mean), _ptr(grad_rotation), _ptr(grad_scale), _ptr(grad_opacity),
                _ptr(grad_color), stream), "gs_project_bwd_views")
            _mark("project_bwd")
        else:
            _mark("begin:project_bwd")
            native.check(lib.gs_project_bwd(
                n, num_sh, _ptr(mean), _ptr(rotation), _ptr(scale), _ptr(opacity), _ptr(color),
                _ptr(camera_rotation), _ptr(camera_translation), _ptr(inverse_covariance),
                _ptr(grad_projected), _ptr(counts), pref, _ptr(grad_mean), _ptr(grad_rotation),
                _ptr(grad_scale), _ptr(grad_opacity), _ptr(grad_color), stream),
                "gs_project_bwd")
            _mark("project_bwd")
    gradients = (grad_mean, grad_rotation, grad_scale, grad_opacity, grad_color)
    return (*gradients, *(None,) * (19 - len(gradients)))


torch.library.register_autograd(
    "gaussian_splats::rasterize", _backward, setup_context=_setup_context
)


def rasterize_outputs(
    splats,
    camera: Camera,
    tile_size: int = 4,
    opacity_threshold: float = 0.999,
    near: float = 0.2,
    far: float = 100.0,
    rendering_mode: Literal["gaussian", "ellipsoid"] = "gaussian",
    confidence: float = 0.95,
    indices: torch.Tensor | None = None,
) -> tuple[torch.Tensor, ...]:
    """All ten operator outputs for ``splats`` seen by ``camera``."""
    fx, fy = camera.focal_length
    cx, cy = camera.principal_point
    image_width, image_height = camera.image_size
    assert tile_size > 0 and tile_size & (tile_size - 1) == 0
    assert image_width % tile_size == 0 and image_height % tile_size == 0
    mean, rotation, scale, opacity, color = (
        splats.mean, splats.rotation, splats.scale, splats.opacity, splats.color,
    )
    if indices is not None:
        mean, rotation, scale, opacity, color = (
            mean[indices], rotation[indices], scale[indices], opacity[indices], color[indices],
        )
    return torch.ops.gaussian_splats.rasterize(
        mean, rotation, scale, opacity, color,
        _to_device(camera.rotation_matrix, mean.device),
        _to_device(camera.translation, mean.device),
        float(fx), float(fy), float(cx), float(cy), int(image_width), int(image_height),
        int(tile_size), float(opacity_threshold), float(near), float(far), rendering_mode,
        float(confidence),
    )


def rasterize(
    splats,
    camera: Camera,
    tile_size: int = 4,
    opacity_threshold: float = 0.999,
    near: float = 0.2,
    far: float = 100.0,
    rendering_mode: Literal["gaussian", "ellipsoid"] = "gaussian",
    confidence: float = 0.95,
    indices: torch.Tensor | None = None,
    backend: str | None = None,
) -> torch.Tensor:
    """Render ``splats`` to an ``[H, W, 3]`` float image.

    Signature of the reference's ``splats.rasterize.rasterize``
    (splats/rasterize.py:12-43) and ``kernels.rasterize.interface.rasterize``
    (interface.py:247-303). ``backend`` exists for call-site compatibility:
    ``None``, ``"b200"`` and ``"triton"`` (the reference's name for the kernel
    path this library replaces) all run the B200 kernels; anything else raises
    ``ValueError`` like the reference's dispatch.
    """
    if backend not in (None, "b200", "triton"):
        raise ValueError(f"Unknown rasterization backend: {backend}")
    return rasterize_outputs(splats, camera, tile_size, opacity_threshold, near, far,
                             rendering_mode, confidence, indices)[0]


def rasterize_batch(
    splats,
    cameras: list[Camera],
    tile_size: int = 4,
    opacity_threshold: float = 0.999,
    near: float = 0.2,
    far: float = 100.0,
    rendering_mode: Literal["gaussian", "ellipsoid"] = "gaussian",
    confidence: float = 0.95,
) -> list[tuple[torch.Tensor, ...]]:
    """Forward render of one scene from several cameras (no autograd).

    Returns, per camera, the ten outputs of ``gaussian_splats::rasterize`` --
    bit-identical to rendering that camera alone. The work is shared where
    views allow it: one launch projects every Gaussian into up to 16 cameras
    (its parameters are read once, the view-independent terms computed once);
    the binning count phases of all views run back to back with one host wait
    for all their intersection totals (instead of one wait per view); then
    every view's sort and compositing are enqueued without further waits.
    The reference renders one camera per call (visualize/gaussian/backend.py:48).
    """
    mean, rotation, scale, opacity, color = map(
        _f32, (splats.mean.detach(), splats.rotation.detach(), splats.scale.detach(),
               splats.opacity.detach(), splats.color.detach()))
    _check_inputs(mean, color, rendering_mode)
    assert tile_size > 0 and tile_size & (tile_size - 1) == 0
    lib = native.lib()
    device = mean.device
    n, num_sh, views = mean.shape[0], color.shape[1], len(cameras)
    if views == 0:
        return []
    params = (native.Params * views)()
    rotations = torch.empty((views, 3, 3), dtype=torch.float32)
    translations = torch.empty((views, 3), dtype=torch.float32)
    sizes = []
    for v, camera in enumerate(cameras):
        fx, fy = camera.focal_length
        cx, cy = camera.principal_point
        width, height = camera.image_size
        assert width % tile_size == 0 and height % tile_size == 0
        params[v] = native.make_params(float(fx), float(fy), float(cx), float(cy), int(width),
                                       int(height), tile_size, opacity_threshold, near, far,
                                       rendering_mode, confidence)
        rotations[v] = camera.rotation_matrix.detach().float().cpu()
        translations[v] = camera.translation.detach().float().cpu()
        sizes.append((int(width), int(height)))
    with torch.cuda.device(device), torch.no_grad():
        stream = _stream(device)
        projected_mean = mean.new_empty((views, n, 3))
        inverse_covariance = mean.new_empty((views, n, 2, 2))
        projected_color = mean.new_empty((views, n, 3))
        projected_opacity = mean.new_empty((views, n, 1))
        bounds = torch.empty((views, n, 4), dtype=torch.int32, device=device)
        counts = torch.empty((views, n), dtype=torch.int32, device=device)
        records = mean.new_empty((views, n, 16))
        native.check(lib.gs_project_fwd_batch(
            n, num_sh, views, _ptr(mean), _ptr(rotation), _ptr(scale), _ptr(opacity),
            _ptr(color), ctypes.c_void_p(rotations.data_ptr()),
            ctypes.c_void_p(translations.data_ptr()), params, _ptr(projected_mean),
            _ptr(inverse_covariance), _ptr(projected_color), _ptr(projected_opacity),
            _ptr(bounds), _ptr(counts), _ptr(records), stream), "gs_project_fwd_batch")

        count_bytes = lib.gs_bin_count_workspace_size(n)
        count_ws = torch.empty((views, count_bytes), dtype=torch.uint8, device=device)
        stride = count_ws.stride(0)
        if stride % 256:
            raise RuntimeError("gaussian_splats_b200: count workspace rows are not 256-byte "
                               "aligned")
        totals = torch.zeros(views, dtype=torch.int64).pin_memory()
        errors = torch.zeros(views, dtype=torch.int32).pin_memory()
        for v in range(views):
            native.check(lib.gs_bin_count_async(
                n, _ptr(projected_mean[v]), _ptr(counts[v]), _ptr(count_ws[v]), count_bytes,
                ctypes.c_void_p(totals.data_ptr() + 8 * v),
                ctypes.c_void_p(errors.data_ptr() + 4 * v), stream), "gs_bin_count_async")
        torch.cuda.current_stream(device).synchronize()
        outputs = []
        for v in range(views):
            if int(errors[v]):
                native.check(-6, "gs_bin_count_async")
            total = int(totals[v])
            if total >= 1 << 30:
                native.check(-3, "gs_bin_count_async")
            width, height = sizes[v]
            num_tiles = (width // tile_size) * (height // tile_size)
            pref = ctypes.byref(params[v])
            gaussian_ids = torch.empty((total,), dtype=torch.int32, device=device)
            ranges = torch.empty((num_tiles, 2), dtype=torch.int64, device=device)
            sort_bytes = lib.gs_bin_sort_workspace_size(n, total, pref)
            sort_ws = torch.empty((sort_bytes,), dtype=torch.uint8, device=device)
            native.check(lib.gs_bin_sort(
                n, total, _ptr(bounds[v]), _ptr(counts[v]), pref, _ptr(count_ws[v]),
                count_bytes, _ptr(sort_ws), sort_bytes, _ptr(gaussian_ids), _ptr(ranges),
                stream), "gs_bin_sort")
            image = mean.new_empty((height, width, 3))
            final_transmittance = mean.new_empty((height, width))
            n_contributors = torch.empty((height, width), dtype=torch.int32, device=device)
            order = _tile_order(ranges, None, pref, stream)
            native.check(lib.gs_composite_fwd(
                _ptr(records[v]), _ptr(gaussian_ids), _ptr(ranges), pref, _ptr(image),
                _ptr(final_transmittance), _ptr(n_contributors), _ptr(order), stream),
                "gs_composite_fwd")
            outputs.append((image, final_transmittance, n_contributors, projected_mean[v],
                            inverse_covariance[v], projected_color[v], projected_opacity[v],
                            gaussian_ids, ranges, counts[v]))
    return outputs
