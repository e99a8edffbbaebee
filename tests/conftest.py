"""Shared test setup.

Markers: ``gpu`` tests need a CUDA device and the built kernel library; the
rest run on CPU (oracle against golden vectors, host logic, library exports,
gloo multi-process paths).
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for path in (ROOT, os.path.join(ROOT, "oracle")):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and libgs_b200.so")


def golden_cases(kind: str = "all") -> list[str]:
    """Golden ``.npz`` case names; ``kind`` = all | backward | rasterize."""
    import numpy as np

    names = sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz"))
    out = []
    for name in names:
        if name in ("adam_noise", "relocate"):  # training-step fixtures (optim, relocate tests)
            continue
        if name == "intersections":
            if kind == "all":
                out.append(name)
            continue
        if kind == "backward":
            with np.load(os.path.join(GOLDEN, name + ".npz")) as d:
                if "grad_mean" not in d.files:
                    continue
        out.append(name)
    return out


@pytest.fixture(scope="session")
def oracle():
    import oracle as O

    O.build()
    return O


def assert_ids_match_up_to_ties(got, expected, depths, ranges):
    """``gaussian_ids`` equal, except that runs of equal (tile, depth bits) may
    be permuted. This build orders such ties by Gaussian index (a stable sort);
    the reference's ``torch.sort`` (intersections.py:82) is not stable, so its
    tie order is unspecified. Returns the number of tied runs seen."""
    import numpy as np

    got = np.asarray(got)
    expected = np.asarray(expected)
    assert got.shape == expected.shape
    bits = np.asarray(depths, dtype=np.float32).view(np.uint32)
    tile_of = np.zeros(len(got), np.int64)
    for t, (start, end) in enumerate(np.asarray(ranges)):
        tile_of[start:end] = t
    key_got = (tile_of << 32) | bits[got].astype(np.int64)
    key_exp = (tile_of << 32) | bits[expected].astype(np.int64)
    np.testing.assert_array_equal(key_got, key_exp, err_msg="(tile, depth) key sequence")
    ties = 0
    if len(got):
        boundaries = np.nonzero(np.diff(key_got))[0] + 1
        for run_g, run_e in zip(np.split(got, boundaries), np.split(expected, boundaries)):
            if len(run_g) > 1:
                ties += 1
                assert sorted(run_g.tolist()) == sorted(run_e.tolist())
            else:
                assert run_g[0] == run_e[0]
    return ties


PARAM_NAMES = ("mean", "rotation", "scale", "opacity", "color")
OUTPUT_NAMES = ("image", "final_transmittance", "n_contributors", "projected_mean",
                "inverse_covariance", "projected_color", "projected_opacity", "gaussian_ids",
                "ranges", "counts")


def run_operator(inputs, settings, grad_image=None, device="cuda"):
    """Runs ``torch.ops.gaussian_splats.rasterize`` on numpy inputs (and, with
    ``grad_image``, its backward); returns numpy outputs and parameter grads."""
    import numpy as np
    import torch

    import gaussian_splats_b200.rasterize  # noqa: F401  registers the operator

    params = [torch.from_numpy(np.ascontiguousarray(inputs[k])).to(device) for k in PARAM_NAMES]
    if grad_image is not None:
        for p in params:
            p.requires_grad_(True)
    s = settings
    out = torch.ops.gaussian_splats.rasterize(
        *params, torch.from_numpy(inputs["camera_rotation"]).to(device),
        torch.from_numpy(inputs["camera_translation"]).to(device), float(s.fx), float(s.fy),
        float(s.cx), float(s.cy), int(s.width), int(s.height), int(s.tile_size),
        float(s.opacity_threshold), float(s.near), float(s.far), s.rendering_mode,
        float(s.confidence))
    result = {k: v.detach().cpu().numpy() for k, v in zip(OUTPUT_NAMES, out)}
    if grad_image is not None:
        torch.autograd.backward(out[0], torch.from_numpy(np.ascontiguousarray(grad_image)).to(device))
        for k, p in zip(PARAM_NAMES, params):
            result["grad_" + k] = p.grad.cpu().numpy()
    torch.cuda.synchronize()
    return result


def scene_inputs(scene, view=0):
    """Numpy operator inputs and oracle settings of a ``scenes.Scene`` view."""
    import oracle as O

    return O.scene_inputs(scene, view)


def l1_grad_image(image, target, crop):
    """d mean|image[:h,:w] - target| / d image, zero in the padding."""
    import numpy as np

    w, h = crop
    g = np.zeros_like(image)
    diff = image[:h, :w] - target
    g[:h, :w] = np.sign(diff) / np.float32(diff.size)
    return g.astype(np.float32)


INPUTS_ORDER = PARAM_NAMES + ("camera_rotation", "camera_translation")


def run_binning(bounds, depths, counts, tiles_w, tiles_h, tile_size=4):
    """gs_bin_count + gs_bin_sort through the C ABI on the GPU; numpy in/out.
    Bounds are in tiles; the image is tiles_w x tiles_h tiles of tile_size."""
    import ctypes

    import numpy as np
    import torch

    from gaussian_splats_b200 import native

    lib = native.lib()
    n = len(counts)
    pm = np.zeros((n, 3), np.float32)
    pm[:, 2] = depths
    d_pm = torch.from_numpy(pm).cuda()
    d_counts = torch.from_numpy(np.ascontiguousarray(counts, np.int32)).cuda()
    d_bounds = torch.from_numpy(np.ascontiguousarray(bounds, np.int32).reshape(n, 4)).cuda()
    params = native.make_params(1.0, 1.0, 0.0, 0.0, tiles_w * tile_size, tiles_h * tile_size,
                                tile_size, 0.999, 0.2, 100.0, "gaussian", 0.95)
    num_tiles = tiles_w * tiles_h
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ptr = lambda t: ctypes.c_void_p(t.data_ptr() if t.numel() else 0)  # noqa: E731
    cbytes = lib.gs_bin_count_workspace_size(n)
    cws = torch.empty(cbytes, dtype=torch.uint8, device="cuda")
    total = ctypes.c_int64(-1)
    native.check(lib.gs_bin_count(n, ptr(d_pm), ptr(d_counts), ptr(cws), cbytes,
                                  ctypes.byref(total), stream), "gs_bin_count")
    total = total.value
    ids = torch.empty(total, dtype=torch.int32, device="cuda")
    ranges = torch.empty((num_tiles, 2), dtype=torch.int64, device="cuda")
    sbytes = lib.gs_bin_sort_workspace_size(n, total, ctypes.byref(params))
    sws = torch.empty(sbytes, dtype=torch.uint8, device="cuda")
    native.check(lib.gs_bin_sort(n, total, ptr(d_bounds), ptr(d_counts), ctypes.byref(params),
                                 ptr(cws), cbytes, ptr(sws), sbytes, ptr(ids), ptr(ranges),
                                 stream), "gs_bin_sort")
    native.check(lib.gs_bin_check(ptr(cws), ptr(sws), stream), "gs_bin_check")
    return total, ids.cpu().numpy(), ranges.cpu().numpy()
