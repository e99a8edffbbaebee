"""Batched multi-camera forward (rasterize_batch): every camera's ten outputs
are bit-identical to rendering that camera alone with the operator."""

import math

import pytest
import torch

from gaussian_splats_b200 import scenes
from gaussian_splats_b200.rasterize import rasterize_batch, rasterize_outputs
from gaussian_splats_b200.splats import GaussianSplat

pytestmark = pytest.mark.gpu


def _orbit(views, sizes):
    cams = []
    for i in range(views):
        angle = 2 * math.pi * i / views
        w, h = sizes[i % len(sizes)]
        cams.append(scenes.look_at_camera((4 * math.cos(angle), 1.0, 4 * math.sin(angle)),
                                          fovy_degrees=55.0, width=w, height=h))
    return cams


@pytest.mark.parametrize("views,sizes,mode,sh", [
    (3, [(128, 64)], "gaussian", 3),
    (20, [(128, 64), (96, 96), (64, 32)], "gaussian", 3),  # two launches of the batch kernel
    (5, [(64, 64)], "ellipsoid", 1),
    (17, [(32, 32)], "gaussian", 4),
])
def test_batch_bit_identical_to_single_views(views, sizes, mode, sh):
    g = torch.Generator().manual_seed(views)
    tensors = scenes.random_gaussians(g, 20_000, means=("normal", 0.0, 1.0), log_scale=(-4.0, 0.7),
                                      opacity_logit=(0.0, 1.5), sh_degree=sh)
    splats = GaussianSplat.from_tensors(*(t.cuda() for t in tensors))
    cameras = _orbit(views, sizes)
    batch = rasterize_batch(splats, cameras, tile_size=16, rendering_mode=mode, near=0.2)
    assert len(batch) == views
    for camera, got in zip(cameras, batch):
        want = rasterize_outputs(splats, camera, tile_size=16, rendering_mode=mode, near=0.2)
        for a, b in zip(got, want):
            assert a.dtype == b.dtype and a.shape == b.shape
            assert torch.equal(a, b)
    assert any(int(out[7].numel()) > 0 for out in batch)
