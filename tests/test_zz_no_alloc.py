"""gs_bin_noalloc: binning for callers that cannot allocate device memory.

Plugins and bindings inside a host program that owns every device allocation,
and per-frame loops that cannot take cudaMalloc's device-wide synchronisation,
have no workspace to pass to gs_bin_count / gs_bin_sort. gs_bin_noalloc does
the same work out of a fixed 64 MiB array inside the library. This checks,
through the C ABI, that two calls in a row (on different scenes, so the second
call starts from the first call's leftovers in the shared array) give exactly
the ids and ranges of the regular entry points -- the tolerance for integer
outputs is zero -- and that inputs beyond the limit are refused with
GS_ERR_CAPACITY. The file is named to be collected last.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GS_ERR_CAPACITY = -3


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None and t.numel() else 0)


def _project(lib, native, scene):
    """gs_project_fwd of the scene's first camera: projected means, counts, bounds."""
    camera = scene.cameras[0]
    fx, fy = camera.focal_length
    cx, cy = camera.principal_point
    w, h = camera.image_size
    st = scene.settings
    params = native.make_params(fx, fy, cx, cy, w, h, st.tile_size, st.opacity_threshold,
                                st.near, st.far, st.rendering_mode, st.confidence)
    mean, rotation, scale, opacity, color = (t.contiguous().cuda() for t in scene.tensors())
    n, k = mean.shape[0], color.shape[1]
    cam_r = camera.rotation_matrix.contiguous().cuda()
    cam_t = camera.translation.contiguous().cuda()
    pm = torch.empty((n, 3), device="cuda")
    conic = torch.empty((n, 4), device="cuda")
    rgb = torch.empty((n, 3), device="cuda")
    o = torch.empty((n, 1), device="cuda")
    bounds = torch.empty((n, 4), dtype=torch.int32, device="cuda")
    counts = torch.empty((n,), dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    native.check(lib.gs_project_fwd(n, k, _ptr(mean), _ptr(rotation), _ptr(scale), _ptr(opacity),
                                    _ptr(color), _ptr(cam_r), _ptr(cam_t), ctypes.byref(params),
                                    _ptr(pm), _ptr(conic), _ptr(rgb), _ptr(o), _ptr(bounds),
                                    _ptr(counts), stream), "gs_project_fwd")
    return params, pm, counts, bounds


def _regular(lib, native, params, pm, counts, bounds):
    n = counts.numel()
    num_tiles = (params.width // params.tile_size) * (params.height // params.tile_size)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    cbytes = lib.gs_bin_count_workspace_size(n)
    cws = torch.empty(cbytes, dtype=torch.uint8, device="cuda")
    total = ctypes.c_int64(0)
    native.check(lib.gs_bin_count(n, _ptr(pm), _ptr(counts), _ptr(cws), cbytes,
                                  ctypes.byref(total), stream), "gs_bin_count")
    ids = torch.empty(total.value, dtype=torch.int32, device="cuda")
    ranges = torch.empty((num_tiles, 2), dtype=torch.int64, device="cuda")
    sbytes = lib.gs_bin_sort_workspace_size(total.value, num_tiles)
    sws = torch.empty(sbytes, dtype=torch.uint8, device="cuda")
    native.check(lib.gs_bin_sort(n, total.value, _ptr(bounds), _ptr(counts), ctypes.byref(params),
                                 _ptr(cws), cbytes, _ptr(sws), sbytes, _ptr(ids), _ptr(ranges),
                                 stream), "gs_bin_sort")
    return ids.cpu().numpy(), ranges.cpu().numpy()


def _noalloc(lib, native, params, pm, counts, bounds, capacity):
    n = counts.numel()
    num_tiles = (params.width // params.tile_size) * (params.height // params.tile_size)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ids = torch.full((capacity,), -1, dtype=torch.int32, device="cuda")
    ranges = torch.full((num_tiles, 2), -1, dtype=torch.int64, device="cuda")
    total = ctypes.c_int64(-1)
    status = lib.gs_bin_noalloc(n, _ptr(pm), _ptr(counts), _ptr(bounds), ctypes.byref(params),
                                _ptr(ids), capacity, _ptr(ranges), ctypes.byref(total), stream)
    torch.cuda.synchronize()
    return status, total.value, ids.cpu().numpy()[: max(total.value, 0)], ranges.cpu().numpy()


def test_noalloc_matches_regular_binning_twice_in_a_row():
    from gaussian_splats_b200 import native, scenes

    lib = native.lib()
    scene_a = scenes.config2(num_points=20_000, width=256, height=144, log_scale=(-3.5, 0.7))
    scene_b = scenes.config5(num_points=6_000, width=128, height=100)
    for scene in (scene_a, scene_b):
        params, pm, counts, bounds = _project(lib, native, scene)
        ref_ids, ref_ranges = _regular(lib, native, params, pm, counts, bounds)
        assert len(ref_ids) > 0
        status, total, ids, ranges = _noalloc(lib, native, params, pm, counts, bounds,
                                              capacity=len(ref_ids) + 17)
        native.check(status, "gs_bin_noalloc")
        assert total == len(ref_ids)
        np.testing.assert_array_equal(ids, ref_ids)
        np.testing.assert_array_equal(ranges, ref_ranges)


def test_noalloc_refuses_what_does_not_fit():
    from gaussian_splats_b200 import native, scenes

    lib = native.lib()
    scene = scenes.config2(num_points=5_000, width=128, height=72, log_scale=(-3.5, 0.7))
    params, pm, counts, bounds = _project(lib, native, scene)
    expected = int(counts.sum())
    # Output buffer smaller than the intersection total: refused, total reported.
    status, total, _, _ = _noalloc(lib, native, params, pm, counts, bounds, capacity=expected - 1)
    assert status == GS_ERR_CAPACITY and total == expected
    # More Gaussians than the 64 MiB scratch can bin: refused before any GPU work.
    n_big = 4_000_000
    total = ctypes.c_int64(-1)
    status = lib.gs_bin_noalloc(n_big, None, None, None, ctypes.byref(params), None, 0, None,
                                ctypes.byref(total), None)
    assert status == GS_ERR_CAPACITY
