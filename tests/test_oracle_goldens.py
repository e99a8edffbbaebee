"""The CPU oracle against golden vectors from the reference's own kernels.

Every ``tests/golden/*.npz`` was produced by running the reference's Triton
rasterizer (``gaussian_splats::rasterize``, forward and autograd backward)
under Triton's CPU interpreter; ``tests/golden/make_goldens.py`` regenerates
them. This pins the oracle that the GPU tests then compare against.

Bars: integer outputs (tile counts, sorted ids, ranges, contributor counts)
bit-exact; projected floats and the image within 1e-5 absolute (the north
star's RGB bar), final transmittance within 1e-5 absolute; parameter
gradients within 1e-4 relative / 1e-6 absolute.
"""

import os

import numpy as np
import pytest

from conftest import GOLDEN, assert_ids_match_up_to_ties, golden_cases

PARAMS = ("mean", "rotation", "scale", "opacity", "color")
INPUTS = PARAMS + ("camera_rotation", "camera_translation")
INT_OUTPUTS = ("counts", "ranges", "n_contributors")
FLOAT_OUTPUTS = ("projected_mean", "projected_color", "projected_opacity", "image",
                 "final_transmittance")


def _run(oracle, name):
    inputs, settings, expected = oracle.load_golden(os.path.join(GOLDEN, name + ".npz"))
    out = oracle.rasterize(*(inputs[k] for k in INPUTS), settings)
    return inputs, settings, expected, out


@pytest.mark.parametrize("name", golden_cases("rasterize"))
def test_forward_integers_exact(oracle, name):
    _, _, expected, out = _run(oracle, name)
    for key in INT_OUTPUTS:
        np.testing.assert_array_equal(out[key], expected["out_" + key], err_msg=key)
    assert_ids_match_up_to_ties(out["gaussian_ids"], expected["out_gaussian_ids"],
                                out["projected_mean"][:, 2], out["ranges"])


@pytest.mark.parametrize("name", golden_cases("rasterize"))
def test_forward_floats(oracle, name):
    _, _, expected, out = _run(oracle, name)
    for key in FLOAT_OUTPUTS:
        np.testing.assert_allclose(out[key], expected["out_" + key], rtol=0, atol=1e-5,
                                   err_msg=key)
    # The conic is the inverse of a 2x2 covariance whose determinant cancels;
    # compare relative to each Gaussian's largest conic entry.
    got, ref = out["inverse_covariance"], expected["out_inverse_covariance"]
    scale = np.abs(ref).reshape(len(ref), -1).max(axis=1)[:, None, None]
    worst = float((np.abs(got - ref) / (scale + 1e-30)).max()) if len(ref) else 0.0
    assert worst < 1e-4, worst


@pytest.mark.parametrize("name", golden_cases("backward"))
def test_backward_gradients(oracle, name):
    inputs, settings, expected, out = _run(oracle, name)
    grads = oracle.backward(inputs, out, inputs["grad_image"], settings)
    for key in PARAMS:
        np.testing.assert_allclose(grads[key], expected["grad_" + key], rtol=1e-4, atol=1e-6,
                                   err_msg=key)


def test_intersections_exact(oracle):
    """The reference's random-bounds emit/sort case (test_intersections.py:8-38)."""
    d = np.load(os.path.join(GOLDEN, "intersections.npz"))
    tiles_w, tiles_h = (int(v) for v in d["in_tiles"])
    s = oracle.Settings(fx=1, fy=1, cx=0, cy=0, width=tiles_w, height=tiles_h, tile_size=1)
    out = oracle.bin(d["in_bounds"], d["in_depths"], d["in_counts"], s, with_keys=True)
    np.testing.assert_array_equal(out["keys"], d["out_keys"])
    np.testing.assert_array_equal(out["ids"], d["out_ids"])
    np.testing.assert_array_equal(out["gaussian_ids"], d["out_sorted_ids"])
    np.testing.assert_array_equal(out["ranges"], d["out_ranges"])
    depths = d["in_depths"]
    for start, end in out["ranges"]:
        tile_depths = depths[out["gaussian_ids"][start:end]]
        assert np.all(tile_depths[:-1] <= tile_depths[1:])


def test_goldens_are_not_degenerate():
    """Each rendering golden except the stock-camera one has visible Gaussians
    and pixels that reach the opacity threshold somewhere."""
    for name in golden_cases("rasterize"):
        d = np.load(os.path.join(GOLDEN, name + ".npz"))
        visible = int((d["out_counts"] > 0).sum())
        if name == "fixture_degenerate":
            assert visible == 0
            continue
        assert visible > 0, name
        assert d["out_image"].max() > 0.05, name
