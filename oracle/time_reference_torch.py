"""Times the reference's own pure-PyTorch rasterizer on this host's CPU cores
-- TEST INFRASTRUCTURE, run only where the reference checkout is mounted.

The reference (VikaasVarma/gaussian-splats) is Python; its CPU path is
``kernels/rasterize/torch.py:228-247`` (project -> cull -> tile -> render).
It cannot travel to the GPU box, so this measures it here, on the seeded
config scenes the benchmark uses, and prints one JSON line per case:

* config 1 (16,384 Gaussians, 256x256): the whole view, forward (no_grad)
  and forward + L1-loss backward;
* config 2 (1M Gaussians, 1920x1088): ``render`` needs O(intersections x 256)
  intermediates, beyond host memory for a whole 1080p view, so ``project``,
  ``cull`` and ``tile`` run on the whole scene and ``render`` over bands of
  tile rows, each band's list re-based and the band images summed (exactly
  the whole image: every tile belongs to one band). For fwd+bwd (timed
  unless ``--forward-only``) the band losses' gradients w.r.t. the projected
  tensors are accumulated and back-propagated through project once.
  Labelled "band-summed".

Times are the median of ``--repeats`` runs after one warm-up, with
``torch.set_num_threads(<all host cores>)``.

    PYTHONDONTWRITEBYTECODE=1 TORCHDYNAMO_DISABLE=1 \\
        python oracle/time_reference_torch.py --reference <checkout> [--config 1|2]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def reference_objects(ref, scene):
    """The reference's GaussianSplat and PinholeCamera holding the scene's
    tensors and its first camera."""
    import torch

    mean, rotation, scale, opacity, color = scene.tensors()
    degree = int(round(color.shape[1] ** 0.5)) - 1
    splats = ref.GaussianSplat(mean.shape[0], sh_degree=degree)
    with torch.no_grad():
        for name, value in zip(("mean", "rotation", "scale", "opacity", "color"),
                               (mean, rotation, scale, opacity, color)):
            getattr(splats, name).copy_(value)
    cam = scene.cameras[0]
    camera = ref.PinholeCamera(rotation=cam.rotation.clone(), translation=cam.translation.clone(),
                               image_size=tuple(cam.image_size),
                               focal_length=tuple(cam.focal_length),
                               principal_point=tuple(cam.principal_point))
    return splats, camera


def l1(image, target):
    height, width = target.shape[:2]
    return (image[:height, :width] - target).abs().mean()


def whole_view(ref, splats, camera, settings, target, backward):
    import torch

    kw = dict(tile_size=settings.tile_size, opacity_threshold=settings.opacity_threshold,
              near=settings.near, far=settings.far)
    if not backward:
        with torch.no_grad():
            ref.rasterize(splats, camera, **kw)
        return
    splats.zero_grad(set_to_none=True)
    l1(ref.rasterize(splats, camera, **kw), target).backward()


def banded_view(ref, splats, camera, settings, target, backward, band_rows):
    """project/cull/tile on the whole scene, render band by band (summed)."""
    import torch

    T = ref.T
    ts = settings.tile_size
    width, height = camera.image_size
    tiles_w, tiles_h = width // ts, height // ts
    context = torch.enable_grad() if backward else torch.no_grad()
    with context:
        if backward:
            splats.zero_grad(set_to_none=True)
        projected = T.project(splats, camera)
        projected = T.cull(projected, settings.near, settings.far)
        indices, ranges = T.tile(projected, camera, ts)
        leaves = projected
        if backward:
            # render's inputs as leaves: band gradients accumulate here, then
            # flow through project once
            leaves = ref.ProjectedGaussianSplat(
                projected.mean.detach().requires_grad_(),
                projected.covariance.detach().requires_grad_(),
                projected.color.detach().requires_grad_(),
                projected.opacity.detach().requires_grad_())
        image = torch.zeros(height, width, 3)
        count = target.numel() if target is not None else 1
        for row0 in range(0, tiles_h, band_rows):
            t0, t1 = row0 * tiles_w, min(tiles_h, row0 + band_rows) * tiles_w
            first, last = int(ranges[t0, 0]), int(ranges[t1 - 1, 1])
            band_ranges = torch.zeros_like(ranges)
            band_ranges[t0:t1] = ranges[t0:t1] - first
            band = T.render(leaves, camera, (indices[first:last], band_ranges), ts,
                            settings.opacity_threshold)
            if backward:
                # this band's share of the L1 mean over the cropped image
                rows = slice(row0 * ts, min(tiles_h, row0 + band_rows) * ts)
                crop = band[:target.shape[0], :target.shape[1]][rows]
                # retain_graph: the bands share project's cached inverse covariance
                ((crop - target[rows]).abs().sum() / count).backward(retain_graph=True)
            image += band.detach()
        if backward:
            torch.autograd.backward(
                [projected.mean, projected.covariance, projected.color, projected.opacity],
                [leaves.mean.grad, leaves.covariance.grad, leaves.color.grad,
                 leaves.opacity.grad])
    return image


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--reference", required=True, help="the reference checkout")
    p.add_argument("--config", type=int, choices=(1, 2), default=1)
    p.add_argument("--repeats", type=int, default=3)
    p.add_argument("--band-rows", type=int, default=4, help="tile rows per band (config 2)")
    p.add_argument("--forward-only", action="store_true")
    args = p.parse_args()
    sys.dont_write_bytecode = True
    os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
    sys.path.insert(0, os.path.join(args.reference, "src"))
    sys.path.insert(0, ROOT)
    import torch

    from gaussian_splats.kernels.rasterize import torch as ref_torch
    from gaussian_splats.splats.camera import PinholeCamera
    from gaussian_splats.splats.splats import GaussianSplat, ProjectedGaussianSplat

    import gaussian_splats_b200  # noqa: F401  (the scene generators)
    from gaussian_splats_b200 import scenes

    class Ref:
        T = ref_torch
        rasterize = staticmethod(ref_torch.rasterize)

    Ref.GaussianSplat, Ref.PinholeCamera = GaussianSplat, PinholeCamera
    Ref.ProjectedGaussianSplat = ProjectedGaussianSplat
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    scene = getattr(scenes, f"config{args.config}")()
    splats, camera = reference_objects(Ref, scene)
    settings = scene.settings
    target = None
    if scene.targets:
        target = scene.targets[0]
    else:
        width, height = scene.crop
        target = torch.rand(height, width, 3, generator=torch.Generator().manual_seed(999))
    modes = (False,) if args.forward_only else (False, True)
    for backward in modes:
        if args.config == 1:
            run = lambda: whole_view(Ref, splats, camera, settings, target, backward)  # noqa
            how = "whole view"
        else:
            run = lambda: banded_view(Ref, splats, camera, settings, target, backward,  # noqa
                                      args.band_rows)
            how = f"band-summed ({args.band_rows} tile rows per band)"
        run()  # warm-up
        times = []
        for _ in range(args.repeats):
            t0 = time.perf_counter()
            run()
            times.append(time.perf_counter() - t0)
        print(json.dumps({
            "path": "reference kernels/rasterize/torch.py:228-247 (PyTorch eager, CPU)",
            "config": args.config, "gaussians": scene.num_points, "image": list(scene.crop),
            "tile_size": settings.tile_size, "pass": "fwd+bwd (L1)" if backward else "fwd",
            "how": how, "seconds_median": statistics.median(times), "seconds": times,
            "threads": threads, "torch": torch.__version__}), flush=True)


if __name__ == "__main__":
    main()
