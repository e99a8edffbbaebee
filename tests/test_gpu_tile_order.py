"""The compositors' heavy-first tile order (gs_tile_order): a permutation of
the view's tiles with work classes non-increasing along it (list lengths for
the forward, largest contributor counts for the backward), and compositing
in that order gives the forward's outputs bit for bit and the backward's
gradients within tolerance of the row-major order."""

import ctypes

import numpy as np
import pytest
import torch

from gaussian_splats_b200 import native, scenes
from gaussian_splats_b200.rasterize import rasterize_outputs
from gaussian_splats_b200.splats import GaussianSplat

pytestmark = pytest.mark.gpu


def _work_class(w: int) -> int:
    """The kernel's class of a work amount: 0 for none, else 1 + 4 floor(log2 w)
    + the two bits below the leading one, capped at 63."""
    if w == 0:
        return 0
    b = w.bit_length() - 1
    frac = (w >> (b - 2)) & 3 if b >= 2 else (w << (2 - b)) & 3
    return min(1 + 4 * b + frac, 63)


@pytest.mark.parametrize("tile", [8, 16])
def test_tile_order_is_heavy_first_and_changes_nothing(tile):
    # a dense blob: list lengths span several octaves
    scene = scenes.config5(num_points=20_000, width=320, height=192)
    splats = GaussianSplat.from_tensors(*(t.cuda() for t in scene.tensors()))
    camera = scene.cameras[0]
    out = rasterize_outputs(splats, camera, tile_size=tile)
    image, final_t, n_contrib, pm, conic, rgb, op, ids, ranges, counts = out
    lib = native.lib()
    fx, fy = camera.focal_length
    cx, cy = camera.principal_point
    w, h = camera.image_size
    params = native.make_params(fx, fy, cx, cy, w, h, tile, 0.999, 0.2, 100.0, "gaussian", 0.95)
    pref = ctypes.byref(params)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    num_tiles = ranges.shape[0]
    fwd_order = torch.empty((num_tiles,), dtype=torch.int32, device="cuda")
    bwd_order = torch.empty_like(fwd_order)  # (the deterministic backward's order)
    scratch = torch.empty((num_tiles + 128,), dtype=torch.int32, device="cuda")
    native.check(lib.gs_tile_order(P(ranges), None, pref, P(fwd_order), P(scratch), stream),
                 "order")
    native.check(lib.gs_tile_order(P(ranges), P(n_contrib), pref, P(bwd_order), P(scratch),
                                   stream), "order")
    torch.cuda.synchronize()

    lengths = (ranges[:, 1] - ranges[:, 0]).cpu().tolist()
    tw = w // tile
    nc = n_contrib.cpu().view(h // tile, tile, tw, tile).permute(0, 2, 1, 3).reshape(num_tiles, -1)
    max_contrib = nc.max(1).values.tolist()
    for order, work in ((fwd_order, lengths), (bwd_order, max_contrib)):
        o = order.cpu().tolist()
        assert sorted(o) == list(range(num_tiles))
        classes = [_work_class(int(work[t])) for t in o]
        assert all(a >= b for a, b in zip(classes, classes[1:]))
    assert len({_work_class(int(x)) for x in lengths}) > 4  # the scene exercises the order

    # forward: the same bits in either order
    img2, t2 = torch.empty_like(image), torch.empty_like(final_t)
    nc2 = torch.empty_like(n_contrib)
    records = torch.empty((pm.shape[0], 16), device="cuda")
    n = pm.shape[0]
    native.check(lib.gs_pack_records(n, P(pm), P(conic), P(rgb), P(op), pref, P(records),
                                     stream), "pack")
    for order in (None, P(fwd_order)):
        img2.fill_(float("nan"))
        native.check(lib.gs_composite_fwd(P(records), P(ids), P(ranges), pref, P(img2), P(t2),
                                          P(nc2), order, stream), "fwd")
        torch.cuda.synchronize()
        assert torch.equal(img2, image) and torch.equal(t2, final_t)
        assert torch.equal(nc2, n_contrib)

    # backward: whole tiles in row-major order, the plan's heavy-first items,
    # and plans that split every walk longer than 64 or 8 entries all agree
    # to the gradient tolerance
    grad_image = torch.rand_like(image)
    plan_bytes = lib.gs_composite_bwd_plan_size(pref)
    grads = []
    for split_walk in (None, 0, 64, 8):
        plan = None
        if split_walk is not None:
            plan = torch.empty((plan_bytes,), dtype=torch.uint8, device="cuda")
            native.check(lib.gs_composite_bwd_plan(P(ranges), P(n_contrib), pref, split_walk,
                                                   P(plan), plan_bytes, stream), "plan")
        gp = torch.empty((n, 9), device="cuda")
        native.check(lib.gs_composite_bwd(n, P(records), P(ids), P(ranges), P(grad_image),
                                          P(final_t), P(n_contrib), pref, P(gp),
                                          P(plan) if plan is not None else None, stream),
                     "bwd")
        torch.cuda.synchronize()
        grads.append(gp)
        if split_walk == 8:
            _check_plan(plan, num_tiles, lengths, max_contrib, 8)
    for g in grads[1:]:
        torch.testing.assert_close(g, grads[0], rtol=1e-4, atol=1e-6)


EXTRA_PARTS = 1024  # parts beyond the tiles' first ones that one plan can hold


def _check_plan(plan, num_tiles, lengths, max_contrib, split_walk):
    """Every tile's walk is covered once: one item per part, the parts of a
    split tile numbered 0..parts-1, splits only where the walk is longer than
    split_walk, no more extra parts than the plan holds."""
    words = plan.cpu().numpy().view(np.int32)
    num_items, extra = int(words[0]), int(words[1])
    items = words[256:256 + 4 * (num_tiles + EXTRA_PARTS)].reshape(-1, 4)  # after 1 KB
    live = items[:num_items]
    assert np.all(items[num_items:, 0] == -1)
    walks = np.minimum(np.asarray(lengths), np.asarray(max_contrib))
    seen = {}
    for tile, part, parts, _ in live:
        seen.setdefault(int(tile), []).append((int(part), int(parts)))
    assert sorted(seen) == list(range(num_tiles))
    split_parts = 0
    for tile, entries in seen.items():
        parts = entries[0][1]
        assert sorted(e[0] for e in entries) == list(range(parts))
        assert all(e[1] == parts for e in entries)
        if parts > 1:
            assert walks[tile] > split_walk
            split_parts += parts - 1
    assert 0 < split_parts <= min(extra, EXTRA_PARTS)
