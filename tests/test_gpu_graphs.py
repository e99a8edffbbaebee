"""Steps replayed from CUDA graphs (gaussian_splats_b200.graphs): the same
results as launching them from Python, device cameras updated in place
between replays, and recovery when a new view outgrows the captured
intersection buffer."""

import math

import pytest
import torch

from gaussian_splats_b200 import scenes
from gaussian_splats_b200.graphs import CapturedStep
from gaussian_splats_b200.rasterize import rasterize_outputs
from gaussian_splats_b200.splats import GaussianSplat
from gaussian_splats_b200.view_parallel import train_step

pytestmark = pytest.mark.gpu

W, H = 320, 240


def _scene(n=30_000, seed=4):
    g = torch.Generator().manual_seed(seed)
    tensors = scenes.random_gaussians(g, n, means=("normal", 0.0, 1.0), log_scale=(-4.0, 0.7),
                                      opacity_logit=(0.0, 1.5), sh_degree=3)
    splats = GaussianSplat.from_tensors(*(t.cuda() for t in tensors))
    params = [splats.mean, splats.rotation, splats.scale, splats.opacity, splats.color]
    return splats, params


def _camera(angle, distance=4.0):
    return scenes.look_at_camera((distance * math.cos(angle), 0.5, distance * math.sin(angle)),
                                 fovy_degrees=55.0, width=W, height=H)


def _render(splats, camera):
    return rasterize_outputs(splats, camera, 16)[0]


def test_captured_training_step_matches_eager():
    splats, params = _scene()
    for p in params:
        p.requires_grad_(True)
    camera = _camera(0.3)
    target = torch.rand(H, W, 3, generator=torch.Generator().manual_seed(1)).cuda()

    def loss_fn(image, t):
        return (image - t).abs().mean()

    def fn():
        return train_step(splats, [camera], [target], params, _render, loss_fn)

    eager_loss = fn().clone()
    eager_grads = [p.grad.clone() for p in params]
    step = CapturedStep(fn)
    for _ in range(3):
        loss = step()
    assert step.check() and step.captures == 1
    assert torch.equal(loss, eager_loss)  # the forward is deterministic
    for a, b in zip((p.grad for p in params), eager_grads):
        # compositing backward's float atomics add in scheduling order
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-4 * float(b.abs().max()))


def test_device_camera_updates_in_place_and_overflow_recaptures():
    splats, _ = _scene()
    camera = _camera(0.0).to("cuda")
    with torch.no_grad():
        step = CapturedStep(lambda: _render(splats, camera))
        first = step().clone()
        assert step.check()
        assert torch.equal(first, _render(splats, camera))
        # another direction at the same distance: the captured buffer holds it
        other = _camera(1.2)
        camera.rotation.copy_(other.rotation)
        camera.translation.copy_(other.translation)
        image = step().clone()
        assert step.check() and step.captures == 1
        assert not torch.equal(image, first)
        assert torch.equal(image, _render(splats, camera))
        # splats 2.7x larger (in place, as a training step would change them):
        # more intersections than the capture's buffer holds; the replay is
        # flagged, the step re-captured and replayed
        (_, capacity, _), = step.renders
        splats.scale.data += 1.0
        assert rasterize_outputs(splats, camera, 16)[7].numel() > capacity
        step()
        assert step.check() is False and step.captures == 2
        assert torch.equal(step.output, _render(splats, camera))
        step()
        assert step.check() and step.captures == 2

