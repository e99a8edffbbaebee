"""Full benchmark-size parity: configs 2 (1M Gaussians, 1080p) and 5 (dense
blob, ~57M intersections) at their real sizes.

The oracle checks what it can finish in seconds at this size: projection and
binning of every Gaussian (bit-exact), compositing of a sample of tiles that
includes the longest lists (bit-exact), and gradients of an L1 loss whose
pixel gradient is kept only on the sampled tiles (so the oracle only needs to
walk those tiles; 1e-4 relative / 1e-6 absolute). Size-independent properties
cover the rest of the image: ranges tile the id list, lists are in (depth, id)
order, every listed Gaussian's rectangle covers its tile, transmittance lies
in [0, 1].
"""

import numpy as np
import pytest

from conftest import INPUTS_ORDER, PARAM_NAMES, l1_grad_image, run_operator, scene_inputs

pytestmark = pytest.mark.gpu


def _sample_tiles(ranges, count, seed):
    lengths = ranges[:, 1] - ranges[:, 0]
    longest = np.argsort(lengths)[-count // 2:]
    rng = np.random.default_rng(seed)
    rest = rng.choice(len(ranges), size=count - len(longest), replace=False)
    return np.unique(np.concatenate([longest, rest])).astype(np.int32)


def _tile_mask(settings, tiles):
    ts = settings.tile_size
    tiles_w = settings.width // ts
    mask = np.zeros((settings.height, settings.width), bool)
    for t in tiles:
        y, x = divmod(int(t), tiles_w)
        mask[y * ts:(y + 1) * ts, x * ts:(x + 1) * ts] = True
    return mask


def _check_config(oracle, scene, sample, seed):
    inputs, s = scene_inputs(scene)
    got = run_operator(inputs, s)
    proj = oracle.project(*(inputs[k] for k in INPUTS_ORDER), s)
    for key in ("projected_mean", "inverse_covariance", "projected_color", "projected_opacity",
                "counts"):
        np.testing.assert_array_equal(got[key], proj[key], err_msg=key)
    binned = oracle.bin(proj["bounds"], proj["projected_mean"][:, 2], proj["counts"], s)
    np.testing.assert_array_equal(got["ranges"], binned["ranges"])
    np.testing.assert_array_equal(got["gaussian_ids"], binned["gaussian_ids"])

    # Properties over the whole image.
    ranges, ids = got["ranges"], got["gaussian_ids"]
    assert ranges[0, 0] == 0 and ranges[-1, 1] == len(ids) == int(got["counts"].sum())
    assert np.all(ranges[1:, 0] == ranges[:-1, 1]) and np.all(ranges[:, 1] >= ranges[:, 0])
    tile_of = np.repeat(np.arange(len(ranges)), ranges[:, 1] - ranges[:, 0])
    depth_bits = got["projected_mean"][:, 2].view(np.uint32).astype(np.uint64)
    key = (tile_of.astype(np.uint64) << np.uint64(32)) | depth_bits[ids]
    assert np.all((key[:-1] < key[1:]) | ((key[:-1] == key[1:]) & (ids[:-1] < ids[1:])))
    b = proj["bounds"].reshape(-1, 4)[ids]
    tiles_w = s.width // s.tile_size
    tx, ty = tile_of % tiles_w, tile_of // tiles_w
    assert np.all((b[:, 0] <= tx) & (tx < b[:, 1]) & (b[:, 2] <= ty) & (ty < b[:, 3]))
    T = got["final_transmittance"]
    assert np.all((T >= 0) & (T <= 1)) and np.all(np.isfinite(got["image"]))

    # Exact compositing on sampled tiles.
    tiles = _sample_tiles(ranges, sample, seed)
    comp = oracle.composite(proj["projected_mean"], proj["inverse_covariance"],
                            proj["projected_color"], proj["projected_opacity"], ids, ranges, s,
                            tiles=tiles)
    mask = _tile_mask(s, tiles)
    for key in ("image", "final_transmittance", "n_contributors"):
        np.testing.assert_array_equal(got[key][mask], comp[key][mask], err_msg=key)

    # Gradients with the loss restricted to the sampled tiles.
    grad_image = l1_grad_image(got["image"], scene.targets[0].numpy(), scene.crop)
    grad_image[~mask] = 0.0
    got_b = run_operator(inputs, s, grad_image=grad_image)
    fwd = dict(proj, gaussian_ids=ids, ranges=ranges, **{
        k: got[k] for k in ("image", "final_transmittance", "n_contributors")})
    grads = oracle.backward(inputs, fwd, grad_image, s, tiles=tiles)
    for key in PARAM_NAMES:
        np.testing.assert_allclose(got_b["grad_" + key], grads[key], rtol=1e-4, atol=1e-6,
                                   err_msg=key)
    return got


def test_config2_full_size(oracle):
    from gaussian_splats_b200 import scenes

    got = _check_config(oracle, scenes.config2(), sample=192, seed=0)
    assert len(got["gaussian_ids"]) > 1_000_000


def test_config5_full_size(oracle):
    from gaussian_splats_b200 import scenes

    got = _check_config(oracle, scenes.config5(), sample=64, seed=1)
    lengths = got["ranges"][:, 1] - got["ranges"][:, 0]
    assert lengths.max() > 100_000  # the skewed per-tile lists this config exists for
