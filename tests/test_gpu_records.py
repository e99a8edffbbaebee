"""The compositors' per-Gaussian records: what the projection writes equals
what gs_pack_records rebuilds from the operator's outputs (bit for bit, on
every Gaussian that lands in a tile), and a backward that has to rebuild them
(a second backward of the same render) gives the gradients of the first."""

import ctypes

import pytest
import torch

from gaussian_splats_b200 import native, scenes
from gaussian_splats_b200.rasterize import rasterize_outputs
from gaussian_splats_b200.splats import GaussianSplat

pytestmark = pytest.mark.gpu


def _scene(mode_scale=(-3.5, 0.7)):
    scene = scenes.config2(num_points=30_000, width=256, height=144, log_scale=mode_scale)
    splats = GaussianSplat.from_tensors(*(t.cuda() for t in scene.tensors()))
    return scene, splats


@pytest.mark.parametrize("mode", ["gaussian", "ellipsoid"])
def test_projection_records_equal_packed_records(mode):
    scene, splats = _scene()
    camera = scene.cameras[0]
    lib = native.lib()
    fx, fy = camera.focal_length
    cx, cy = camera.principal_point
    w, h = camera.image_size
    params = native.make_params(fx, fy, cx, cy, w, h, 16, 0.999, 0.2, 100.0, mode, 0.95)
    n, k = splats.mean.shape[0], splats.color.shape[1]
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    pm, conic = torch.empty((n, 3), device="cuda"), torch.empty((n, 4), device="cuda")
    rgb, o = torch.empty((n, 3), device="cuda"), torch.empty((n, 1), device="cuda")
    bounds = torch.empty((n, 4), dtype=torch.int32, device="cuda")
    counts = torch.empty((n,), dtype=torch.int32, device="cuda")
    written = torch.full((n, 16), float("nan"), device="cuda")
    cam_r = camera.rotation_matrix.contiguous().cuda()
    cam_t = camera.translation.contiguous().cuda()
    native.check(lib.gs_project_fwd(n, k, P(splats.mean), P(splats.rotation), P(splats.scale),
                                    P(splats.opacity), P(splats.color), P(cam_r), P(cam_t),
                                    ctypes.byref(params), P(pm), P(conic), P(rgb), P(o),
                                    P(bounds), P(counts), P(written), stream), "project")
    packed = torch.empty((n, 16), device="cuda")
    native.check(lib.gs_pack_records(n, P(pm), P(conic), P(rgb), P(o), ctypes.byref(params),
                                     P(packed), stream), "pack")
    visible = counts > 0
    assert int(visible.sum()) > 1000
    a, b = written[visible], packed[visible]
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))  # NaN-safe bitwise equality
    # the record's index word is the Gaussian's own index
    ids = torch.nonzero(visible).squeeze(1).to(torch.int32)
    assert torch.equal(a[:, 11].view(torch.int32), ids)


def test_second_backward_rebuilds_records():
    scene, splats = _scene()
    params = [splats.mean, splats.rotation, splats.scale, splats.opacity, splats.color]
    for p in params:
        p.requires_grad_(True)
    out = rasterize_outputs(splats, scene.cameras[0], 16)
    weights = torch.randn(out[0].shape, device="cuda",
                          generator=torch.Generator(device="cuda").manual_seed(3))
    loss = (out[0] * weights).sum()
    first = torch.autograd.grad(loss, params, retain_graph=True)  # the forward's records
    second = torch.autograd.grad(loss, params)  # records rebuilt by gs_pack_records
    for a, b in zip(first, second):
        assert torch.count_nonzero(a) > 0
        # float atomics add in scheduling order: tolerance on the tensor's scale
        torch.testing.assert_close(b, a, rtol=1e-4, atol=1e-5 * float(a.abs().max()))
