"""Generate golden vectors by running the reference's own rasterizer.

The reference (VikaasVarma/gaussian-splats) is pure Python; its GPU path is six
Triton kernels wrapped in the ``gaussian_splats::rasterize`` custom op
(kernels/rasterize/interface.py:17-244). Triton's CPU interpreter
(``TRITON_INTERPRET=1``) runs those same kernels without a GPU, so this script
imports the reference from a source checkout, calls the op (forward and, where
the case asks, autograd backward), and writes inputs, all ten op outputs and
the parameter gradients to ``tests/golden/<case>.npz``.

Run it where the reference checkout exists (it is not needed afterwards):

    TRITON_INTERPRET=1 TORCHDYNAMO_DISABLE=1 PYTHONDONTWRITEBYTECODE=1 \
        python tests/golden/make_goldens.py --reference <checkout>/src [case ...]

Scenes:
* ``fixture_*``: the reference's own test fixture (kernels/rasterize/tests/
  common.py:19-50: seed 42, 5 % near-plane, far-plane, off-screen and large
  Gaussians, 32x32, fx = fy = 24), with the camera turned to face +Z so the
  Gaussians are in front of it (the stock fixture's identity camera sees none
  of them; ``fixture_degenerate`` keeps that camera).
* ``mini2`` / ``mini5``: configs 2 and 5 at a few thousand Gaussians and a
  small padded image (96x60 and 64x60), L1 loss against a random target.
* ``config1``: the full config-1 forward (16,384 Gaussians, 256x256).
* ``intersections``: the reference's random-bounds emit/sort case
  (kernels/rasterize/tests/test_intersections.py:8-18).
* ``adam_noise``: the training loop's optimizer step (training/train.py:
  111-118,151: torch.optim.Adam, one group per splat tensor, eps 1e-15, the
  default learning rates) for three steps of random gradients on a
  GaussianSplat of 257 Gaussians, then the reference's own noise_splats
  (training/utils.py:50-62) with a recorded seed; the normal samples it draws
  are stored too.
* ``relocate``: the training loop's splat relocation (training/utils.py:
  120-210): copy_splats with chosen counts, and relocate_splats with an Adam
  optimizer and densification, with the counts it sampled.
"""

from __future__ import annotations

import argparse
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent

OUTPUT_NAMES = (
    "image",
    "final_transmittance",
    "n_contributors",
    "projected_mean",
    "inverse_covariance",
    "projected_color",
    "projected_opacity",
    "gaussian_ids",
    "ranges",
    "counts",
)
PARAM_NAMES = ("mean", "rotation", "scale", "opacity", "color")


def _fixture(sh_degree: int, num_points: int = 1000, face: bool = True):
    from gaussian_splats.kernels.rasterize.tests.common import make_scene

    splats, camera = make_scene(num_points, sh_degree=sh_degree)
    if face:
        # Half turn about +Y: camera axes (-x, y, -z), so world +Z is in front.
        camera.rotation = torch.tensor([0.0, 0.0, 1.0, 0.0])
    tensors = tuple(getattr(splats, n).detach().clone() for n in PARAM_NAMES)
    fx, fy = camera.focal_length
    cx, cy = camera.principal_point
    w, h = camera.image_size
    return tensors, camera.rotation_matrix, camera.translation.clone(), (fx, fy, cx, cy, w, h)


def _from_scene(scene):
    camera = scene.cameras[0]
    fx, fy = camera.focal_length
    cx, cy = camera.principal_point
    w, h = camera.image_size
    return (
        scene.tensors(),
        camera.rotation_matrix,
        camera.translation.clone(),
        (fx, fy, cx, cy, w, h),
    )


def build_case(name: str) -> dict:
    sys.path.insert(0, str(REPO))
    from gaussian_splats_b200 import scenes

    settings = dict(tile_size=8, opacity_threshold=0.999, near=0.1, far=100.0,
                    rendering_mode="gaussian", confidence=0.95)
    crop = None
    target = None
    loss = "square_mean"
    backward = True
    if name == "fixture_sh1_t8":
        tensors, cam_r, cam_t, intr = _fixture(1)
    elif name == "fixture_sh0_t8":
        tensors, cam_r, cam_t, intr = _fixture(0)
        backward = False
    elif name == "fixture_sh4_t8":
        tensors, cam_r, cam_t, intr = _fixture(4)
        backward = False
    elif name == "fixture_sh2_t8":
        tensors, cam_r, cam_t, intr = _fixture(2)
    elif name == "fixture_sh3_t16":
        tensors, cam_r, cam_t, intr = _fixture(3)
        settings["tile_size"] = 16
    elif name == "fixture_sh1_t4":
        tensors, cam_r, cam_t, intr = _fixture(1)
        settings["tile_size"] = 4
    elif name == "fixture_ellipsoid":
        tensors, cam_r, cam_t, intr = _fixture(1)
        settings["rendering_mode"] = "ellipsoid"
        backward = False
    elif name == "fixture_degenerate":
        tensors, cam_r, cam_t, intr = _fixture(1, face=False)
        backward = False
    elif name == "mini2":
        scene = scenes.config2(num_points=3000, width=96, height=60, log_scale=(-3.5, 0.7))
        tensors, cam_r, cam_t, intr = _from_scene(scene)
        settings.update(tile_size=16, near=0.2)
        crop, target, loss = scene.crop, scene.targets[0], "l1"
    elif name == "mini5":
        scene = scenes.config5(num_points=1500, width=64, height=60)
        tensors, cam_r, cam_t, intr = _from_scene(scene)
        settings.update(tile_size=16, near=0.2)
        crop, target, loss = scene.crop, scene.targets[0], "l1"
    elif name == "config1":
        scene = scenes.config1()
        tensors, cam_r, cam_t, intr = _from_scene(scene)
        settings.update(tile_size=16, near=scene.settings.near)
        backward = False
    else:
        raise KeyError(name)
    return dict(tensors=tensors, cam_r=cam_r, cam_t=cam_t, intr=intr, settings=settings,
                crop=crop, target=target, loss=loss, backward=backward)


def run_case(name: str) -> dict:
    import gaussian_splats.kernels.rasterize.interface  # noqa: F401  registers the op

    case = build_case(name)
    tensors = [t.clone().requires_grad_(case["backward"]) for t in case["tensors"]]
    fx, fy, cx, cy, w, h = case["intr"]
    s = case["settings"]
    args = (*tensors, case["cam_r"], case["cam_t"], float(fx), float(fy), float(cx), float(cy),
            int(w), int(h), s["tile_size"], s["opacity_threshold"], s["near"], s["far"],
            s["rendering_mode"], s["confidence"])
    out = torch.ops.gaussian_splats.rasterize(*args)
    record = {}
    for i, t in enumerate(case["tensors"]):
        record["in_" + PARAM_NAMES[i]] = t.numpy()
    record["in_camera_rotation"] = case["cam_r"].numpy()
    record["in_camera_translation"] = case["cam_t"].numpy()
    record["in_intrinsics"] = np.array([fx, fy, cx, cy], dtype=np.float64)
    record["in_image_size"] = np.array([w, h], dtype=np.int64)
    record["in_tile_size"] = np.array(s["tile_size"])
    record["in_opacity_threshold"] = np.array(s["opacity_threshold"])
    record["in_near_far"] = np.array([s["near"], s["far"]])
    record["in_rendering_mode"] = np.array(s["rendering_mode"])
    record["in_confidence"] = np.array(s["confidence"])
    for n, t in zip(OUTPUT_NAMES, out):
        record["out_" + n] = t.detach().numpy()
    if case["backward"]:
        image = out[0]
        if case["loss"] == "l1":
            cw, ch = case["crop"]
            loss = (image[:ch, :cw] - case["target"]).abs().mean()
            record["in_target"] = case["target"].numpy()
            record["in_crop"] = np.array(case["crop"])
        else:
            loss = image.square().mean()
        grad_image = torch.autograd.grad(loss, image, retain_graph=True)[0]
        grads = torch.autograd.grad(image, tensors, grad_image)
        record["in_grad_image"] = grad_image.numpy()
        for n, g in zip(PARAM_NAMES, grads):
            record["grad_" + n] = g.numpy()
    return record


def run_intersections() -> dict:
    """The reference's random-bounds case, through its Triton emit + torch sort."""
    from gaussian_splats.kernels.rasterize.intersections import (
        emit_intersections,
        sort_intersections,
    )

    tiles_w = tiles_h = 8
    with torch.random.fork_rng():
        torch.manual_seed(42)
        corners = torch.randint(0, tiles_w + 1, (256, 2, 2))
        depths = torch.rand(256) * 10.0 + 0.1
    bounds = torch.stack((corners.amin(dim=-1), corners.amax(dim=-1)), dim=-1).to(torch.int32)
    counts = (bounds[:, :, 1] - bounds[:, :, 0]).prod(dim=-1).to(torch.int32)
    keys, ids = emit_intersections(bounds, depths, counts, tiles_w)
    sorted_ids, ranges = sort_intersections(keys, ids, tiles_w * tiles_h)
    return dict(
        in_bounds=bounds.numpy(), in_depths=depths.numpy(), in_counts=counts.numpy(),
        in_tiles=np.array([tiles_w, tiles_h]), out_keys=keys.numpy(), out_ids=ids.numpy(),
        out_sorted_ids=sorted_ids.numpy(), out_ranges=ranges.numpy(),
    )


def _training_utils():
    """The reference's training/utils.py module. It imports torchmetrics (for
    its SSIM, unused here) and the package __init__ pulls in the whole
    training script; neither is needed for the splat helpers. Stub the one and
    skip the other."""
    import importlib
    import types

    import gaussian_splats

    if "torchmetrics" not in sys.modules:
        image = types.ModuleType("torchmetrics.functional.image")
        image.structural_similarity_index_measure = None
        functional = types.ModuleType("torchmetrics.functional")
        functional.image = image
        root = types.ModuleType("torchmetrics")
        root.functional = functional
        sys.modules.update({"torchmetrics": root, "torchmetrics.functional": functional,
                            "torchmetrics.functional.image": image})
    if "gaussian_splats.training" not in sys.modules:
        package = types.ModuleType("gaussian_splats.training")
        package.__path__ = [os.path.join(os.path.dirname(gaussian_splats.__file__), "training")]
        sys.modules["gaussian_splats.training"] = package
    return importlib.import_module("gaussian_splats.training.utils")


def run_adam_noise() -> dict:
    """torch.optim.Adam as the reference's training loop builds it, then its
    noise_splats, on the reference's GaussianSplat."""
    from gaussian_splats.splats.splats import GaussianSplat

    noise_splats = _training_utils().noise_splats

    n, lrs = 257, (1.6e-4 * 3.3, 1e-3, 5e-3, 5e-2, 2.5e-3)  # train.py:78-83 (mean lr scaled)
    noise_lr, position_lr = 5e5, 1.6e-4 * 3.3
    g = torch.Generator().manual_seed(11)
    splats = GaussianSplat(n, sh_degree=3)
    with torch.no_grad():
        splats.mean.copy_(torch.randn(n, 3, generator=g))
        splats.rotation.copy_(torch.randn(n, 4, generator=g))
        splats.scale.copy_(torch.randn(n, 3, generator=g) * 0.5 - 4.0)
        splats.opacity.copy_(torch.randn(n, 1, generator=g) * 3.0 - 4.0)
        splats.color.copy_(torch.randn(n, 16, 3, generator=g) * 0.3)
    params = [splats.mean, splats.rotation, splats.scale, splats.opacity, splats.color]
    record = {f"in_{name}": p.detach().numpy().copy() for name, p in zip(PARAM_NAMES, params)}
    groups = [{"params": [p], "name": name, "lr": lr}
              for p, name, lr in zip(params, PARAM_NAMES, lrs)]
    optimizer = torch.optim.Adam(groups, eps=1e-15)
    for step in range(3):
        for name, p in zip(PARAM_NAMES, params):
            grad = torch.randn(p.shape, generator=g) * 10.0 ** -(1 + step)
            record[f"in_grad{step}_{name}"] = grad.numpy().copy()
            p.grad = grad
        optimizer.step()
        optimizer.zero_grad()
    for name, p in zip(PARAM_NAMES, params):
        record[f"adam_{name}"] = p.detach().numpy().copy()
        state = optimizer.state[p]
        record[f"exp_avg_{name}"] = state["exp_avg"].numpy().copy()
        record[f"exp_avg_sq_{name}"] = state["exp_avg_sq"].numpy().copy()
    torch.manual_seed(1234)
    record["in_randn"] = torch.randn_like(splats.mean).numpy().copy()
    torch.manual_seed(1234)
    noise_splats(splats, noise_lr, position_lr)
    record["noised_mean"] = splats.mean.detach().numpy().copy()
    record["in_lrs"] = np.array(lrs)
    record["in_noise"] = np.array([noise_lr, position_lr])
    return record


def run_relocate() -> dict:
    """The reference's copy_splats and relocate_splats on CPU.

    copy_*: copy_splats (training/utils.py:120-145) with chosen counts -- one
    parent with 55 copies (normalize_copies clamps copies at 51), three with 1
    to 3 -- into 61 non-parent rows listed in random order.
    reloc_*: relocate_splats (training/utils.py:147-210) with a
    torch.optim.Adam that has taken one step, densification factor 1.05 and
    torch seed 5; the counts its sample_counts drew (dead rows, then
    densification) are recorded so a test can replay them."""
    from gaussian_splats.splats.splats import GaussianSplat

    utils = _training_utils()
    names = PARAM_NAMES + ("normals",)
    n = 300
    g = torch.Generator().manual_seed(21)

    def make():
        splats = GaussianSplat(n, sh_degree=1)
        with torch.no_grad():
            splats.mean.copy_(torch.randn(n, 3, generator=g))
            splats.rotation.copy_(torch.randn(n, 4, generator=g))
            splats.scale.copy_(torch.randn(n, 3, generator=g) * 0.5 - 4.0)
            splats.opacity.copy_(torch.randn(n, 1, generator=g) * 2.5 - 2.0)
            splats.color.copy_(torch.randn(n, 4, 3, generator=g) * 0.3)
            splats.normals.copy_(torch.randn(n, 3, generator=g))
        return splats

    record = {}
    splats = make()
    for name in names:
        record[f"copy_in_{name}"] = getattr(splats, name).detach().numpy().copy()
    alive = (splats.opacity.sigmoid().squeeze(-1) >= 0.005).nonzero().squeeze(-1)
    parents = alive[torch.randperm(len(alive), generator=g)[:4]]
    counts = torch.zeros(n, dtype=torch.int64)
    counts[parents] = torch.tensor([55, 1, 2, 3])
    others = torch.ones(n, dtype=torch.bool)
    others[parents] = False
    candidates = others.nonzero().squeeze(-1)
    outputs = candidates[torch.randperm(len(candidates), generator=g)[:61]]
    reset = utils.copy_splats(splats, counts, outputs)
    record["copy_counts"] = counts.numpy()
    record["copy_outputs"] = outputs.numpy()
    record["copy_reset"] = reset.numpy()
    for name in names:
        record[f"copy_out_{name}"] = getattr(splats, name).detach().numpy().copy()

    splats = make()
    params = [getattr(splats, name) for name in PARAM_NAMES]
    optimizer = torch.optim.Adam([{"params": [p], "name": name, "lr": 1e-3}
                                  for p, name in zip(params, PARAM_NAMES)], eps=1e-15)
    for p in params:
        p.grad = torch.randn(p.shape, generator=g) * 0.1
    optimizer.step()
    for name, p in zip(PARAM_NAMES, params):
        record[f"reloc_in_exp_avg_{name}"] = optimizer.state[p]["exp_avg"].numpy().copy()
        record[f"reloc_in_exp_avg_sq_{name}"] = optimizer.state[p]["exp_avg_sq"].numpy().copy()
    for name in names:
        record[f"reloc_in_{name}"] = getattr(splats, name).detach().numpy().copy()
    drawn = []
    sample = utils.sample_counts

    def recording(weights, count):
        out = sample(weights, count)
        drawn.append(out.numpy().copy())
        return out

    utils.sample_counts = recording
    try:
        torch.manual_seed(5)
        utils.relocate_splats(splats, optimizer, densification_factor=1.05)
    finally:
        utils.sample_counts = sample
    assert len(drawn) == 2, "expected a dead-row and a densification draw"
    record["reloc_counts_dead"], record["reloc_counts_densify"] = drawn
    for name in names:
        record[f"reloc_out_{name}"] = getattr(splats, name).detach().numpy().copy()
    for group in optimizer.param_groups:
        state = optimizer.state[group["params"][0]]
        record[f"reloc_out_exp_avg_{group['name']}"] = state["exp_avg"].numpy().copy()
        record[f"reloc_out_exp_avg_sq_{group['name']}"] = state["exp_avg_sq"].numpy().copy()
    return record


CASES = ("relocate", "adam_noise", "intersections", "fixture_degenerate", "fixture_sh1_t8", "fixture_sh0_t8",
         "fixture_sh4_t8", "fixture_sh2_t8", "fixture_ellipsoid", "fixture_sh1_t4",
         "fixture_sh3_t16", "mini5", "mini2", "config1")


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="path to the reference's src/")
    parser.add_argument("cases", nargs="*", default=list(CASES))
    args = parser.parse_args()
    if os.environ.get("TRITON_INTERPRET") != "1":
        raise SystemExit("set TRITON_INTERPRET=1 (the Triton kernels run on the CPU interpreter)")
    sys.path.insert(0, args.reference)
    torch.set_num_threads(os.cpu_count() or 1)
    for name in args.cases:
        t0 = time.time()
        if name == "intersections":
            record = run_intersections()
        elif name == "adam_noise":
            record = run_adam_noise()
        elif name == "relocate":
            record = run_relocate()
        else:
            record = run_case(name)
        np.savez_compressed(HERE / f"{name}.npz", **record)
        print(f"{name}: {time.time() - t0:.1f}s", flush=True)


if __name__ == "__main__":
    main()
