"""Backward paths the reference lacks (SH degree 4; ellipsoid rendering),
checked in the oracle against independent float64 autograd restatements.

The reference's backward stops at SH coefficient 16 (project_bwd.py:33) and
refuses ellipsoid rendering (interface.py:184-186), so there are no reference
gradients to pin these to; the restatements below differentiate the
reference's forward formulas (project.py:10-71 for SH, composite.py:25-107
for compositing) with torch autograd in float64.
"""

import os

import numpy as np
import torch

from conftest import GOLDEN

C = (0.28209479177387814, -0.4886025119029199, 0.4886025119029199, -0.4886025119029199,
     1.0925484305920792, -1.0925484305920792, 0.31539156525252005, -1.0925484305920792,
     0.5462742152960396, -0.5900435899266435, 2.890611442640554, -0.4570457994644658,
     0.3731763325901154, -0.4570457994644658, 1.445305721320277, -0.5900435899266435,
     2.5033429417967046, -1.7701307697799304, 0.9461746957575601, -0.6690465435572892,
     0.10578554691520431, -0.6690465435572892, 0.47308734787878004, -1.7701307697799304,
     0.6258357354491761)


def _sh_basis(d):
    """The 25 real SH basis functions of the forward (project.py:22-61)."""
    x, y, z = d.unbind(-1)
    xx, yy, zz = x * x, y * y, z * z
    one = torch.ones_like(x)
    terms = (one, y, z, x, x * y, y * z, 2 * zz - xx - yy, x * z, xx - yy, y * (3 * xx - yy),
             x * y * z, y * (4 * zz - xx - yy), z * (2 * zz - 3 * xx - 3 * yy),
             x * (4 * zz - xx - yy), z * (xx - yy), x * (xx - 3 * yy), x * y * (xx - yy),
             y * z * (3 * xx - yy), x * y * (7 * zz - 1), y * z * (7 * zz - 3),
             zz * (35 * zz - 30) + 3, x * z * (7 * zz - 3), (xx - yy) * (7 * zz - 1),
             x * z * (xx - 3 * yy), xx * (xx - 3 * yy) - yy * (3 * xx - yy))
    return torch.stack([c * t for c, t in zip(C, terms)], dim=-1)


def test_sh_degree4_vjp_matches_autograd(oracle):
    d = np.load(os.path.join(GOLDEN, "fixture_sh4_t8.npz"))
    inputs, settings, _ = oracle.load_golden(os.path.join(GOLDEN, "fixture_sh4_t8.npz"))
    keys = ("mean", "rotation", "scale", "opacity", "color", "camera_rotation",
            "camera_translation")
    proj = oracle.project(*(inputs[k] for k in keys), settings)
    n = inputs["mean"].shape[0]
    rng = np.random.default_rng(0)
    grad_rgb = rng.standard_normal((n, 3)).astype(np.float32)
    grad_projected = np.zeros((n, 9), np.float32)
    grad_projected[:, 5:8] = grad_rgb  # only the colour path: isolates the SH VJP
    got = oracle.project_bwd(*(inputs[k] for k in keys), proj["inverse_covariance"],
                             grad_projected, proj["counts"], settings)
    mean = torch.tensor(inputs["mean"], dtype=torch.float64, requires_grad=True)
    color = torch.tensor(inputs["color"], dtype=torch.float64, requires_grad=True)
    r = torch.tensor(inputs["camera_rotation"], dtype=torch.float64)
    t = torch.tensor(inputs["camera_translation"], dtype=torch.float64)
    direction = mean + r.T @ t  # the mean seen from the camera centre -R^T t
    basis = _sh_basis(direction / direction.norm(dim=-1, keepdim=True))
    raw = (basis[:, :, None] * color).sum(1) + 0.5
    rgb = raw.clamp_min(0.0)
    visible = torch.tensor(proj["counts"] > 0)[:, None]
    (rgb * torch.tensor(grad_rgb, dtype=torch.float64) * visible).sum().backward()
    assert d["in_color"].shape[1] == 25 and (proj["counts"] > 0).sum() > 100
    np.testing.assert_allclose(got["color"], color.grad.numpy(), rtol=1e-4, atol=1e-6)
    assert np.abs(got["color"][:, 16:]).max() > 1e-3  # degree 4 really has gradients
    np.testing.assert_allclose(got["mean"], mean.grad.numpy(), rtol=1e-3, atol=1e-5)


def _composite_tile_torch(px, py, means, conics, opacities, colors, cutoff, threshold):
    """Front-to-back compositing of one tile in ellipsoid mode
    (composite.py:25-107 with the indicator falloff), float64, autograd."""
    image = []
    for x, y in zip(px, py):
        T = torch.ones((), dtype=torch.float64)
        c = torch.zeros(3, dtype=torch.float64)
        for mean, conic, o, rgb in zip(means, conics, opacities, colors):
            if not (1 - T.item()) < threshold:
                break
            dx, dy = x - mean[0], y - mean[1]
            d2 = conic[0] * dx * dx + 2 * conic[1] * dx * dy + conic[3] * dy * dy
            inside = 1.0 if d2 <= cutoff else 0.0
            alpha = torch.clamp(o * inside, max=0.99)
            if alpha.item() < 1 / 255:
                continue
            c = c + T * alpha * rgb
            T = T * (1 - alpha)
        image.append(c)
    return torch.stack(image)


def test_ellipsoid_backward_matches_autograd(oracle):
    inputs, settings, _ = oracle.load_golden(os.path.join(GOLDEN, "fixture_ellipsoid.npz"))
    assert settings.rendering_mode == "ellipsoid"
    fwd = oracle.rasterize(*(inputs[k] for k in ("mean", "rotation", "scale", "opacity",
                                                 "color", "camera_rotation",
                                                 "camera_translation")), settings)
    lengths = fwd["ranges"][:, 1] - fwd["ranges"][:, 0]
    tile = int(np.argmax(lengths))
    ts, tiles_w = settings.tile_size, settings.width // settings.tile_size
    x0, y0 = (tile % tiles_w) * ts, (tile // tiles_w) * ts
    rng = np.random.default_rng(1)
    grad_image = np.zeros((settings.height, settings.width, 3), np.float32)
    grad_image[y0:y0 + ts, x0:x0 + ts] = rng.standard_normal((ts, ts, 3)).astype(np.float32)
    got = oracle.composite_bwd(fwd, grad_image, settings,
                               tiles=np.array([tile], np.int32))
    ids = fwd["gaussian_ids"][fwd["ranges"][tile, 0]:fwd["ranges"][tile, 1]]
    opac = torch.tensor(fwd["projected_opacity"][ids, 0], dtype=torch.float64,
                        requires_grad=True)
    rgb = torch.tensor(fwd["projected_color"][ids], dtype=torch.float64, requires_grad=True)
    means = torch.tensor(fwd["projected_mean"][ids], dtype=torch.float64, requires_grad=True)
    conics = torch.tensor(fwd["inverse_covariance"][ids].reshape(-1, 4), dtype=torch.float64)
    py, px = np.mgrid[y0:y0 + ts, x0:x0 + ts]
    image = _composite_tile_torch(px.ravel().astype(np.float64), py.ravel().astype(np.float64),
                                  means, conics, opac, rgb, -2 * np.log1p(-settings.confidence),
                                  settings.opacity_threshold)
    weights = torch.tensor(grad_image[y0:y0 + ts, x0:x0 + ts].reshape(-1, 3), dtype=torch.float64)
    (image * weights).sum().backward()
    # several splats listed more than once are summed per Gaussian by the oracle
    expected_o = np.zeros(fwd["projected_opacity"].shape[0])
    expected_c = np.zeros((fwd["projected_opacity"].shape[0], 3))
    np.add.at(expected_o, ids, opac.grad.numpy())
    np.add.at(expected_c, ids, rgb.grad.numpy())
    assert len(ids) > 10 and np.abs(expected_o).max() > 1e-3
    np.testing.assert_allclose(got[:, 8], expected_o, rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(got[:, 5:8], expected_c, rtol=1e-4, atol=1e-6)
    assert np.all(got[:, :5] == 0)  # the indicator has no position/conic gradient
    assert means.grad is None or torch.count_nonzero(means.grad) == 0
