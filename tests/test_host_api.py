"""Host-side API behaviour that needs no GPU: conventions, folding, errors."""

import math

import numpy as np
import pytest
import torch

from gaussian_splats_b200 import native, scenes
from gaussian_splats_b200.camera import PinholeCamera
from gaussian_splats_b200.splats import GaussianSplat
from gaussian_splats_b200.utils import quaternion_from_rotation, quaternion_to_rotation_matrix


def test_params_fold_like_the_reference():
    p = native.make_params(1166.6, 1166.6, 960.0, 540.0, 1920, 1088, 16, 0.999, 0.2, 100.0,
                           "gaussian", 0.95)
    assert p.lim_x == np.float32(1.3 * 120 * 16 / (2.0 * 1166.6))
    assert p.bwd_lim_y == np.float32(1.3 * 1088 / (2.0 * 1166.6))
    assert p.gaussian_mode == 1 and p.extent == 3.0
    e = native.make_params(10.0, 10.0, 8.0, 8.0, 16, 16, 8, 0.999, 0.2, 100.0, "ellipsoid", 0.9)
    assert e.gaussian_mode == 0
    assert e.extent == np.float32(math.sqrt(-2 * math.log1p(-0.9)))
    assert e.cutoff == np.float32(-2.0 * math.log1p(-0.9))


def test_quaternion_round_trip():
    g = torch.Generator().manual_seed(0)
    for _ in range(20):
        q = torch.randn(4, generator=g, dtype=torch.float64)
        q = q / q.norm()
        r = quaternion_to_rotation_matrix(q)
        q2 = quaternion_from_rotation(r)
        assert torch.allclose(quaternion_to_rotation_matrix(q2), r, atol=1e-12)


def test_look_at_camera_conventions():
    cam = scenes.look_at_camera((0.0, 0.0, 4.0), fovy_degrees=60.0, width=256, height=256)
    # Looking down -Z from +Z: the origin projects to the principal point at depth 4.
    p = cam.rotation_matrix @ torch.zeros(3) + cam.translation
    assert torch.allclose(p, torch.tensor([0.0, 0.0, -4.0]), atol=1e-6)
    assert torch.allclose(cam.position, torch.tensor([0.0, 0.0, 4.0]), atol=1e-6)
    assert cam.focal_length[0] == pytest.approx(128 / math.tan(math.radians(30)))


def test_padding_keeps_principal_point_at_unpadded_centre():
    scene = scenes.config2(num_points=10)
    cam = scene.cameras[0]
    assert cam.image_size == (1920, 1088)
    assert cam.principal_point == (960.0, 540.0)
    assert scene.crop == (1920, 1080)


def test_scenes_are_seeded():
    a = scenes.config5(num_points=100)
    b = scenes.config5(num_points=100)
    for x, y in zip(a.tensors(), b.tensors()):
        assert torch.equal(x, y)
    assert a.color.shape == (100, 4, 3)
    c = scenes.config2(num_points=100)
    assert c.color.shape == (100, 16, 3)
    assert torch.allclose(c.rotation.norm(dim=-1), torch.ones(100), atol=1e-6)


def test_checkpoint_round_trip(tmp_path):
    splats = GaussianSplat(50, sh_degree=2)
    path = tmp_path / "s.pt"
    splats.save_checkpoint(path)
    loaded = GaussianSplat.from_checkpoint(path)
    assert loaded.sh_degree == 2
    for key, value in splats.state_dict().items():
        assert torch.equal(value, loaded.state_dict()[key])


def test_cpu_tensors_are_rejected_not_rendered():
    import gaussian_splats_b200.rasterize as R

    splats = GaussianSplat(10, sh_degree=0)
    camera = PinholeCamera(image_size=(16, 16), focal_length=(10.0, 10.0),
                           principal_point=(8.0, 8.0))
    with torch.no_grad(), pytest.raises(RuntimeError, match="no CPU fallback"):
        R.rasterize(splats, camera, tile_size=8)


def test_wrapper_argument_errors():
    import gaussian_splats_b200.rasterize as R

    splats = GaussianSplat(10, sh_degree=0)
    camera = PinholeCamera(image_size=(16, 16), focal_length=(10.0, 10.0),
                           principal_point=(8.0, 8.0))
    with pytest.raises(AssertionError):
        R.rasterize(splats, camera, tile_size=3)
    with pytest.raises(AssertionError):
        R.rasterize(splats, camera, tile_size=32)
    with pytest.raises(ValueError, match="backend"):
        R.rasterize(splats, camera, tile_size=8, backend="torch")


def test_batch_has_no_cpu_path():
    from gaussian_splats_b200.rasterize import rasterize_batch

    splats = GaussianSplat(10, sh_degree=0)
    camera = PinholeCamera(image_size=(16, 16), focal_length=(10.0, 10.0),
                           principal_point=(8.0, 8.0))
    with pytest.raises(RuntimeError, match="no CPU"):
        rasterize_batch(splats, [camera], tile_size=8)
