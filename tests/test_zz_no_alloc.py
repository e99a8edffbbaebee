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
                                    _ptr(counts), None, stream), "gs_project_fwd")
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
    sbytes = lib.gs_bin_sort_workspace_size(n, total.value, ctypes.byref(params))
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


SCRATCH_BYTES = 64 << 20  # the library's fixed scratch array


def _synthetic_tiles(n, tiles_w, tiles_h, total, seed):
    """n Gaussians as the binning reads them -- depths, per-Gaussian tile
    counts and tile rectangles with count == area -- whose counts add up to
    exactly `total`: some rectangles cover the whole grid, the others are
    random and rows of 1 x w rectangles take up the remainder."""
    rng = np.random.default_rng(seed)
    grid = tiles_w * tiles_h
    full = max(0, (total - 24 * n) // grid)  # whole-grid rectangles
    m = n - full
    widths = rng.integers(1, 17, m)
    heights = rng.integers(1, 9, m)
    heights[::2] = 1  # half the rows stay one tile high, to take the remainder
    area = widths * heights
    rest = total - full * grid
    # Scale the random rectangles down until they leave room for the rest.
    keep = np.cumsum(area) <= rest - (m - np.arange(1, m + 1))
    widths[~keep], heights[~keep] = 1, 1
    remainder = rest - int((widths * heights).sum())
    row = 0
    while remainder > 0:  # widen single-row rectangles, up to a full row each
        if heights[row] == 1:
            add = min(remainder, tiles_w - int(widths[row]))
            widths[row] += add
            remainder -= add
        row += 1
    widths = np.concatenate([widths, np.full(full, tiles_w)])
    heights = np.concatenate([heights, np.full(full, tiles_h)])
    order = rng.permutation(n)
    widths, heights = widths[order], heights[order]
    assert int((widths * heights).sum()) == total
    x0 = rng.integers(0, tiles_w - widths + 1)
    y0 = rng.integers(0, tiles_h - heights + 1)
    bounds = np.stack([x0, x0 + widths, y0, y0 + heights], 1).astype(np.int32)
    counts = (widths * heights).astype(np.int32)
    pm = np.zeros((n, 3), np.float32)
    pm[:, 2] = rng.uniform(0.5, 50.0, n).astype(np.float32)
    return (torch.from_numpy(pm).cuda(), torch.from_numpy(counts).cuda(),
            torch.from_numpy(bounds).cuda())


def test_noalloc_limit_is_the_documented_scratch_size():
    """Just under the 64 MiB limit (count-phase scratch for n Gaussians plus
    sort-phase scratch for the total, as the workspace-size queries report
    them) the call is accepted and matches the regular path; one intersection
    more is refused with GS_ERR_CAPACITY and the total still reported."""
    from gaussian_splats_b200 import native

    lib = native.lib()
    n, tile, tiles_w, tiles_h = 100_000, 16, 64, 64
    params = native.make_params(500.0, 500.0, 512.0, 512.0, tiles_w * tile, tiles_h * tile,
                                tile, 0.999, 0.2, 100.0, "gaussian", 0.95)
    num_tiles = tiles_w * tiles_h
    count_bytes = (lib.gs_bin_count_workspace_size(n) + 255) // 256 * 256

    def fits(t):
        return (count_bytes + lib.gs_bin_sort_workspace_size(n, t, ctypes.byref(params))
                <= SCRATCH_BYTES)

    lo, hi = 0, SCRATCH_BYTES // 4
    while lo + 1 < hi:  # largest total that fits
        mid = (lo + hi) // 2
        lo, hi = (mid, hi) if fits(mid) else (lo, mid)
    limit = lo
    assert fits(limit) and not fits(limit + 1)
    # ~18 B per Gaussian, then ~4.3 B per intersection at 64x64 tiles (the
    # row/column path's segment array and pass-B status)
    assert 14_000_000 < limit < 16_500_000

    pm, counts, bounds = _synthetic_tiles(n, tiles_w, tiles_h, limit, seed=5)
    ref_ids, ref_ranges = _regular(lib, native, params, pm, counts, bounds)
    assert len(ref_ids) == limit
    status, total, ids, ranges = _noalloc(lib, native, params, pm, counts, bounds,
                                          capacity=limit)
    native.check(status, "gs_bin_noalloc at its limit")
    assert total == limit
    np.testing.assert_array_equal(ids, ref_ids)
    np.testing.assert_array_equal(ranges, ref_ranges)

    pm, counts, bounds = _synthetic_tiles(n, tiles_w, tiles_h, limit + 1, seed=6)
    status, total, _, _ = _noalloc(lib, native, params, pm, counts, bounds,
                                   capacity=limit + 1)
    assert status == GS_ERR_CAPACITY and total == limit + 1
