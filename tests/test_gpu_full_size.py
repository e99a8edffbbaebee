"""Full benchmark-size parity: configs 2 (1M Gaussians, 1080p), 3 (3M
Gaussians, 1600x1064), 4 (6M Gaussians, 4K, the batched 16-camera forward)
and 5 (dense blob, ~57M intersections) at their real sizes.

The oracle checks what it can finish in seconds at this size: projection and
binning of every Gaussian (bit-exact), compositing of a sample of tiles that
includes the longest lists (bit-exact), and gradients of an L1 loss whose
pixel gradient is kept only on the sampled tiles (so the oracle only needs to
walk those tiles; 1e-4 relative / 1e-6 absolute). Size-independent properties
cover the rest of the image: ranges tile the id list, lists are in (depth, id)
order, every listed Gaussian's rectangle covers its tile, transmittance lies
in [0, 1]. Where the oracle composites the whole view in seconds (configs 2
and 3) the whole image, transmittance and contributor counts are compared
too. Config 4 checks its batched launch: every one of 16 cameras' ten outputs
bit-identical to rendering that camera alone, and the first camera against
the oracle as above (forward only: config 4 has no backward).
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


def _check_config(oracle, scene, sample, seed, whole_image=False, backward=True):
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
    if whole_image:
        comp = oracle.composite(proj["projected_mean"], proj["inverse_covariance"],
                                proj["projected_color"], proj["projected_opacity"], ids, ranges,
                                s)
        for key in ("image", "final_transmittance", "n_contributors"):
            np.testing.assert_array_equal(got[key], comp[key], err_msg="whole view " + key)
    if not backward:
        return got

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

    got = _check_config(oracle, scenes.config2(), sample=192, seed=0, whole_image=True)
    assert len(got["gaussian_ids"]) > 1_000_000


def test_config3_full_size(oracle):
    from gaussian_splats_b200 import scenes

    scene = scenes.config3()
    assert scene.num_points == 3_000_000 and scene.crop == (1600, 1064)
    got = _check_config(oracle, scene, sample=128, seed=2, whole_image=True)
    assert len(got["gaussian_ids"]) > 3_000_000


def test_config4_batched_full_size(oracle):
    """The bench's config-4 launch shape: 16 cameras of the 4K orbit per
    rasterize_batch call over 6M Gaussians."""
    import torch

    from gaussian_splats_b200 import scenes
    from gaussian_splats_b200.rasterize import rasterize_batch, rasterize_outputs
    from gaussian_splats_b200.splats import GaussianSplat

    scene = scenes.config4()
    assert scene.num_points == 6_000_000 and scene.crop == (3840, 2160)
    splats = GaussianSplat.from_tensors(*(t.cuda() for t in scene.tensors()))
    cameras = scene.cameras[:16]
    st = scene.settings
    with torch.no_grad():
        batch = rasterize_batch(splats, cameras, st.tile_size, st.opacity_threshold, st.near,
                                st.far)
        for camera, got in zip(cameras, batch):
            want = rasterize_outputs(splats, camera, st.tile_size, st.opacity_threshold,
                                     st.near, st.far)
            for name, a, b in zip(("image", "final_transmittance", "n_contributors",
                                   "projected_mean", "inverse_covariance", "projected_color",
                                   "projected_opacity", "gaussian_ids", "ranges", "counts"),
                                  got, want):
                assert a.dtype == b.dtype and a.shape == b.shape, name
                assert torch.equal(a, b), name
            del want
    first = batch[0]
    del batch, splats
    torch.cuda.empty_cache()
    got = _check_config(oracle, scene, sample=96, seed=3, backward=False)
    assert np.array_equal(got["image"], first[0].cpu().numpy())


def test_config5_full_size(oracle):
    from gaussian_splats_b200 import scenes

    got = _check_config(oracle, scenes.config5(), sample=64, seed=1)
    lengths = got["ranges"][:, 1] - got["ranges"][:, 0]
    assert lengths.max() > 100_000  # the skewed per-tile lists this config exists for
