"""ctypes binding of ``libgs_b200.so`` (the C ABI in ``include/gs_b200.h``).

The library is built in-tree by ``__graft_entry__.build()`` (or ``make -C
gaussian-splats_b200/csrc``). There is no fallback: if the library is missing
or fails to load, :func:`lib` raises, and so does every rasterizer call.
"""

from __future__ import annotations

import ctypes
import math
import os

PACKAGE_DIR = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(PACKAGE_DIR, "libgs_b200.so")

GS_OK = 0
STATUS_NAMES = {
    -1: "GS_ERR_INVALID_ARGUMENT",
    -2: "GS_ERR_CUDA",
    -3: "GS_ERR_CAPACITY",
    -4: "GS_ERR_UNSUPPORTED",
    -5: "GS_ERR_MISALIGNED",
    -6: "GS_ERR_TIMEOUT",
}

# Every symbol include/gs_b200.h declares.
EXPORTED_SYMBOLS = (
    "gs_version",
    "gs_last_cuda_error",
    "gs_project_fwd",
    "gs_project_fwd_batch",
    "gs_pack_records",
    "gs_bin_count",
    "gs_bin_count_async",
    "gs_bin_count_workspace_size",
    "gs_bin_sort",
    "gs_bin_sort_workspace_size",
    "gs_bin_check",
    "gs_bin_noalloc",
    "gs_tile_order",
    "gs_composite_fwd",
    "gs_composite_bwd",
    "gs_composite_bwd_plan_size",
    "gs_composite_bwd_plan",
    "gs_composite_bwd_deterministic",
    "gs_composite_bwd_deterministic_workspace_size",
    "gs_project_bwd",
    "gs_project_bwd_views",
    "gs_adam_step",
    "gs_exchange_layout_for",
    "gs_exchange_begin",
    "gs_exchange_publish",
    "gs_exchange_gather",
    "gs_project_bwd_peers",
    "gs_exchange_finish",
    "gs_exchange_status",
    "gs_exchange_shard_layout",
    "gs_exchange_gather_rows",
    "gs_project_bwd_shard",
    "gs_exchange_publish_shard",
    "gs_exchange_gather_shards",
    "gs_l1_loss_scratch_floats",
    "gs_l1_loss",
    "gs_l1_loss_backward",
    "gs_relocate",
    "gs_relocate_status",
    "gs_relocate_workspace_size",
    "gs_det_exp",
    "gs_det_log",
)


class Params(ctypes.Structure):
    """``gs_params`` (include/gs_b200.h)."""

    _fields_ = [
        ("fx", ctypes.c_float), ("fy", ctypes.c_float), ("cx", ctypes.c_float),
        ("cy", ctypes.c_float), ("width", ctypes.c_int32), ("height", ctypes.c_int32),
        ("tile_size", ctypes.c_int32), ("gaussian_mode", ctypes.c_int32),
        ("near_plane", ctypes.c_float), ("far_plane", ctypes.c_float),
        ("lim_x", ctypes.c_float), ("lim_y", ctypes.c_float),
        ("bwd_lim_x", ctypes.c_float), ("bwd_lim_y", ctypes.c_float),
        ("extent", ctypes.c_float), ("cutoff", ctypes.c_float),
        ("opacity_threshold", ctypes.c_float),
    ]


def make_params(fx, fy, cx, cy, width, height, tile_size, opacity_threshold, near, far,
                rendering_mode, confidence) -> Params:
    """Fold the op's scalars like the reference folds its Triton constexprs.

    ``lim_x``/``lim_y`` (project.py:158-159), the backward limits
    (project_bwd.py:376-377), the ellipsoid extent (project.py:308) and cutoff
    (composite.py:226) are evaluated in Python double and rounded to float32.
    """
    tiles_w = width // tile_size
    tiles_h = height // tile_size
    ellipsoid = rendering_mode == "ellipsoid"
    return Params(
        fx=fx, fy=fy, cx=cx, cy=cy, width=width, height=height, tile_size=tile_size,
        gaussian_mode=0 if ellipsoid else 1, near_plane=near, far_plane=far,
        lim_x=1.3 * tiles_w * tile_size / (2.0 * fx),
        lim_y=1.3 * tiles_h * tile_size / (2.0 * fy),
        bwd_lim_x=1.3 * width / (2.0 * fx),
        bwd_lim_y=1.3 * height / (2.0 * fy),
        extent=math.sqrt(-2 * math.log1p(-confidence)) if ellipsoid else 3.0,
        cutoff=-2.0 * math.log1p(-confidence),
        opacity_threshold=opacity_threshold,
    )


class SplatArrays(ctypes.Structure):
    """``gs_splat_arrays``: device pointers of mean, rotation, scale, opacity,
    color (NULL members allowed in a gradient set)."""

    _fields_ = [(name, ctypes.c_void_p) for name in
                ("mean", "rotation", "scale", "opacity", "color")]


GS_MAX_PEERS = 8  # ranks of one peer exchange (include/gs_b200.h)


class PeerGroup(ctypes.Structure):
    """``gs_peer_group``: this rank, the number of ranks, and every rank's
    exchange arena as mapped in this process."""

    _fields_ = [("rank", ctypes.c_int32), ("world", ctypes.c_int32),
                ("arena", ctypes.c_void_p * GS_MAX_PEERS)]


class ExchangeLayout(ctypes.Structure):
    """``gs_exchange_layout``: byte offsets inside an exchange arena."""

    _fields_ = [(name, ctypes.c_uint64) for name in
                ("grad_projected", "counts", "record", "gathered", "bytes")]


class ShardLayout(ctypes.Structure):
    """``gs_shard_layout``: the shard of parameter gradients inside a sharded
    exchange arena (byte offsets), the arena size, and Gaussians per shard."""

    _fields_ = [(name, ctypes.c_uint64) for name in
                ("rotation", "color", "mean", "scale", "opacity", "bytes")] + [
        ("rows", ctypes.c_int64)]


class AdamParams(ctypes.Structure):
    """``gs_adam_params``: one Adam step's scalars (see :func:`adam_params`)."""

    _fields_ = [(name, ctypes.c_float) for name in
                ("lerp_weight", "beta2", "sq_weight", "eps")] + [
        ("neg_step_size", ctypes.c_float * 5), ("bias2_sqrt", ctypes.c_float * 5),
        ("noise_lr", ctypes.c_float), ("position_lr", ctypes.c_float)]


def adam_params(steps, lrs, betas, eps, noise_lr=0.0, position_lr=0.0) -> AdamParams:
    """Fold one Adam step for the five groups (mean, rotation, scale, opacity,
    color) with step numbers ``steps`` (1-based) and learning rates ``lrs`` the
    way torch.optim.Adam's foreach path folds them, in double: bias
    corrections ``1 - beta ** step``, step size ``-(lr / bc1)``, ``sqrt(bc2)``."""
    beta1, beta2 = betas
    h = AdamParams()
    h.lerp_weight, h.beta2, h.sq_weight, h.eps = 1 - beta1, beta2, 1 - beta2, eps
    for k, (step, lr) in enumerate(zip(steps, lrs)):
        bc1 = 1 - beta1 ** step
        bc2 = 1 - beta2 ** step
        h.neg_step_size[k] = (lr / bc1) * -1
        h.bias2_sqrt[k] = bc2 ** 0.5
    h.noise_lr, h.position_lr = noise_lr, position_lr
    return h


VIEW_RECORD_WORDS = 29  # gs_params (17 words) + camera rotation (9) + translation (3)


def view_record(params: Params, camera_rotation, camera_translation, keep=None):
    """The 29-word record of one view for ``gs_project_bwd_views``: the
    render's ``gs_params`` bytes, then the camera rotation and translation as
    float32 (an int32 tensor holding those bits), on the camera tensors'
    device. For CUDA cameras the record is assembled on the device without a
    host wait: the parameter words go up from pinned memory (non-blocking),
    the camera words are concatenated on the device. ``keep``, if given, is
    called with the pinned host buffer the copy reads (a CUDA-graph capture
    must keep it alive and unchanged for as long as the graph replays)."""
    import torch

    device = camera_rotation.device
    header = torch.empty(ctypes.sizeof(Params) // 4, dtype=torch.int32,
                         pin_memory=device.type == "cuda")
    ctypes.memmove(header.data_ptr(), ctypes.addressof(params), ctypes.sizeof(Params))
    if keep is not None:
        keep(header)
    camera = torch.cat((camera_rotation.detach().reshape(9).float(),
                        camera_translation.detach().reshape(3).to(device).float()))
    return torch.cat((header.to(device, non_blocking=True), camera.view(torch.int32)))


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded kernel library; raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIBRARY_PATH):
        raise RuntimeError(
            f"gaussian_splats_b200: {LIBRARY_PATH} is missing; build it with "
            "`python -c 'import __graft_entry__ as g; g.build()'` or "
            "`make -C gaussian-splats_b200/csrc` (there is no CPU fallback)"
        )
    handle = ctypes.CDLL(LIBRARY_PATH)
    vp, i32, i64, u64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64
    P = ctypes.POINTER(Params)
    sigs = {
        "gs_version": ([], i32),
        "gs_last_cuda_error": ([], i32),
        "gs_project_fwd": ([i64, i32] + [vp] * 7 + [P] + [vp] * 7 + [vp], i32),
        "gs_project_fwd_batch": ([i64, i32, i32] + [vp] * 7 + [P] + [vp] * 7 + [vp], i32),
        "gs_pack_records": ([i64] + [vp] * 4 + [P, vp, vp], i32),
        "gs_bin_count": ([i64, vp, vp, vp, u64, ctypes.POINTER(i64), vp], i32),
        "gs_bin_count_async": ([i64, vp, vp, vp, u64, vp, vp, vp], i32),
        "gs_bin_count_workspace_size": ([i64], u64),
        "gs_bin_sort": ([i64, i64, vp, vp, P, vp, u64, vp, u64, vp, vp, vp], i32),
        "gs_bin_sort_workspace_size": ([i64, i64, P], u64),
        "gs_bin_check": ([vp, vp, vp], i32),
        "gs_bin_noalloc": ([i64, vp, vp, vp, P, vp, i64, vp, ctypes.POINTER(i64), vp], i32),
        "gs_tile_order": ([vp, vp, P, vp, vp, vp], i32),
        "gs_composite_fwd": ([vp] * 3 + [P] + [vp] * 4 + [vp], i32),
        "gs_composite_bwd": ([i64] + [vp] * 6 + [P, vp, vp, vp], i32),
        "gs_composite_bwd_plan_size": ([P], u64),
        "gs_composite_bwd_plan": ([vp, vp, P, i32, vp, u64, vp], i32),
        "gs_composite_bwd_deterministic": ([i64, i64] + [vp] * 6 + [P, vp, u64, vp, vp, vp],
                                           i32),
        "gs_composite_bwd_deterministic_workspace_size": ([i64, i64], u64),
        "gs_project_bwd": ([i64, i32] + [vp] * 10 + [P] + [vp] * 5 + [vp], i32),
        "gs_project_bwd_views": ([i64, i32, i32] + [vp] * 13 + [vp], i32),
        "gs_adam_step": ([i64, i32] + [ctypes.POINTER(SplatArrays)] * 4 +
                         [ctypes.POINTER(AdamParams), vp, vp], i32),
        "gs_exchange_layout_for": ([i64, i32, ctypes.POINTER(ExchangeLayout)], i32),
        "gs_exchange_begin": ([ctypes.POINTER(PeerGroup), vp], i32),
        "gs_exchange_publish": ([ctypes.POINTER(PeerGroup), i64, vp], i32),
        "gs_exchange_gather": ([ctypes.POINTER(PeerGroup), i64, vp, vp, vp], i32),
        "gs_project_bwd_peers": ([i64, i32, ctypes.POINTER(PeerGroup)] + [vp] * 12 + [vp], i32),
        "gs_exchange_finish": ([ctypes.POINTER(PeerGroup), vp], i32),
        "gs_exchange_status": ([ctypes.POINTER(PeerGroup), vp], i32),
        "gs_exchange_shard_layout": ([i64, i32, i32, ctypes.POINTER(ShardLayout)], i32),
        "gs_exchange_gather_rows": ([ctypes.POINTER(PeerGroup), i64, vp, vp, vp], i32),
        "gs_project_bwd_shard": ([i64, i32, ctypes.POINTER(PeerGroup)] + [vp] * 7 + [vp], i32),
        "gs_exchange_publish_shard": ([ctypes.POINTER(PeerGroup), vp], i32),
        "gs_exchange_gather_shards": ([ctypes.POINTER(PeerGroup), i64, i32] + [vp] * 5 + [vp],
                                      i32),
        "gs_l1_loss_scratch_floats": ([], i64),
        "gs_l1_loss": ([vp, i64, i64, i64, vp, i64, i64, vp, vp, vp], i32),
        "gs_l1_loss_backward": ([vp, i64, i64, i64, vp, i64, i64, vp, vp, vp], i32),
        "gs_relocate": ([i64, i64, i32, vp, i64, vp, i64, ctypes.POINTER(SplatArrays), vp,
                         ctypes.POINTER(SplatArrays), ctypes.POINTER(SplatArrays), vp,
                         ctypes.c_uint64, vp], i32),
        "gs_relocate_status": ([vp, vp], i32),
        "gs_relocate_workspace_size": ([i64], ctypes.c_uint64),
        "gs_det_exp": ([i64, vp, vp, vp], i32),
        "gs_det_log": ([i64, vp, vp, vp], i32),
    }
    for name, (args, res) in sigs.items():
        fn = getattr(handle, name)
        fn.argtypes = args
        fn.restype = res
    if handle.gs_version() != 100:
        raise RuntimeError(f"gaussian_splats_b200: unexpected library version {handle.gs_version()}")
    _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    """Raise ``RuntimeError`` for a non-zero status from the library."""
    if status == GS_OK:
        return
    name = STATUS_NAMES.get(status, str(status))
    detail = ""
    if status == -2:
        detail = f" (cudaError {lib().gs_last_cuda_error()})"
    raise RuntimeError(f"gaussian_splats_b200: {what} failed with {name}{detail}")
