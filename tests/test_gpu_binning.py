"""Tile binning through the C ABI (gs_bin_count + gs_bin_sort) against the
oracle's restatement of the reference's emit + stable key sort
(intersections.py:10-88). Bit-exact: ids, ranges and the intersection total."""

import os

import numpy as np
import pytest

from conftest import GOLDEN, run_binning

pytestmark = pytest.mark.gpu


def _oracle_bin(oracle, bounds, depths, counts, tiles_w, tiles_h):
    s = oracle.Settings(fx=1, fy=1, cx=0, cy=0, width=tiles_w, height=tiles_h, tile_size=1)
    return oracle.bin(bounds, depths, counts, s)


def _check(oracle, bounds, depths, counts, tiles_w, tiles_h, tile_size=4):
    total, ids, ranges = run_binning(bounds, depths, counts, tiles_w, tiles_h, tile_size)
    ref = _oracle_bin(oracle, bounds, depths, counts, tiles_w, tiles_h)
    assert total == len(ref["gaussian_ids"]) == int(np.asarray(counts, np.int64).sum())
    np.testing.assert_array_equal(ids, ref["gaussian_ids"])
    np.testing.assert_array_equal(ranges, ref["ranges"])
    return ids, ranges


def _random_case(rng, n, tiles_w, tiles_h, max_extent=None, ties=False, culled=0.0):
    x0 = rng.integers(0, tiles_w, n)
    y0 = rng.integers(0, tiles_h, n)
    ex = max_extent or tiles_w
    x1 = np.minimum(x0 + rng.integers(1, ex + 1, n), tiles_w)
    y1 = np.minimum(y0 + rng.integers(1, (max_extent or tiles_h) + 1, n), tiles_h)
    bounds = np.stack([x0, x1, y0, y1], axis=1).astype(np.int32)
    counts = ((x1 - x0) * (y1 - y0)).astype(np.int32)
    if culled:
        counts[rng.random(n) < culled] = 0
    depths = rng.uniform(0.1, 10.0, n).astype(np.float32)
    if ties:
        depths = np.round(depths, 1).astype(np.float32)  # many exact ties
    return bounds, depths, counts


def test_reference_random_bounds_case(oracle):
    """The reference's own test input (test_intersections.py:8-18)."""
    d = np.load(os.path.join(GOLDEN, "intersections.npz"))
    tiles_w, tiles_h = (int(v) for v in d["in_tiles"])
    total, ids, ranges = run_binning(d["in_bounds"], d["in_depths"], d["in_counts"],
                                     tiles_w, tiles_h)
    np.testing.assert_array_equal(ids, d["out_sorted_ids"])
    np.testing.assert_array_equal(ranges, d["out_ranges"])


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_random(oracle, seed):
    rng = np.random.default_rng(seed)
    _check(oracle, *_random_case(rng, 5000, 40, 30, max_extent=6, culled=0.3), 40, 30)


def test_depth_ties_are_stable(oracle):
    rng = np.random.default_rng(3)
    ids, ranges = _check(oracle, *_random_case(rng, 20000, 16, 16, max_extent=4, ties=True),
                         16, 16)
    assert len(ids) > 0


def test_large_footprints(oracle):
    """Gaussians covering most of the screen (config-5-like skew)."""
    rng = np.random.default_rng(4)
    bounds, depths, counts = _random_case(rng, 300, 120, 68)
    bounds[:50] = [0, 120, 0, 68]
    counts[:50] = 120 * 68
    _check(oracle, bounds, depths, counts, 120, 68)


def test_single_tile_and_tile_sizes(oracle):
    rng = np.random.default_rng(5)
    b, d, c = _random_case(rng, 1000, 1, 1)
    _check(oracle, b, d, c, 1, 1)
    b, d, c = _random_case(rng, 1000, 4, 8, max_extent=2)
    _check(oracle, b, d, c, 4, 8, tile_size=16)
    _check(oracle, b, d, c, 4, 8, tile_size=32)


def test_nothing_visible(oracle):
    rng = np.random.default_rng(6)
    b, d, c = _random_case(rng, 777, 8, 8)
    c[:] = 0
    ids, ranges = _check(oracle, b, d, c, 8, 8)
    assert len(ids) == 0 and np.all(ranges == 0)


def test_empty_input(oracle):
    total, ids, ranges = run_binning(np.zeros((0, 4), np.int32), np.zeros(0, np.float32),
                                     np.zeros(0, np.int32), 8, 8)
    assert total == 0 and len(ids) == 0 and np.all(ranges == 0)


def test_million_gaussians(oracle):
    """Many CTAs per pass: exercises the decoupled look-back across ~250 tiles."""
    rng = np.random.default_rng(7)
    b, d, c = _random_case(rng, 1_000_000, 120, 68, max_extent=3, culled=0.05)
    ids, ranges = _check(oracle, b, d, c, 120, 68)
    # Size-independent properties: per-tile depth order, every id in its tile.
    tile_of = np.repeat(np.arange(len(ranges)), ranges[:, 1] - ranges[:, 0])
    keys = (tile_of.astype(np.uint64) << np.uint64(32)) | d[ids].view(np.uint32).astype(np.uint64)
    assert np.all(keys[:-1] <= keys[1:])


def test_negative_depths_sort_like_unsigned_bits(oracle):
    """A negative near plane lets negative depths through; the reference's key
    keeps their raw float bits (intersections.py:27,38), so within a tile they
    sort after every positive depth. Same here."""
    rng = np.random.default_rng(8)
    b, d, c = _random_case(rng, 3000, 8, 8, max_extent=3)
    d[::3] *= -1.0
    _check(oracle, b, d, c, 8, 8)


@pytest.mark.parametrize("tiles_w,tiles_h", [
    (240, 135),   # a 4K view at 16x16 tiles: row/column path
    (256, 512),   # the largest grid the row/column path takes
    (257, 6),     # one tile column too many for its tables: radix path
    (32, 513),    # one tile row too many: radix path
])
def test_grid_shapes_and_both_paths(oracle, tiles_w, tiles_h):
    """Both sort-phase paths (row/column scatter; emit + tile radix sort) and
    the edges between them give the same bit-exact lists."""
    rng = np.random.default_rng(tiles_w * 7 + tiles_h)
    b, d, c = _random_case(rng, 40000, tiles_w, tiles_h, max_extent=12, culled=0.1)
    ids, ranges = _check(oracle, b, d, c, tiles_w, tiles_h)
    assert len(ids) > 0


def test_one_row_many_segments(oracle):
    """Every Gaussian in one tile row: one row's segments span many pass-B
    chunks, whose look-back runs within the row."""
    rng = np.random.default_rng(9)
    b, d, c = _random_case(rng, 200_000, 120, 1, max_extent=5)
    _check(oracle, b, d, c, 120, 1)
