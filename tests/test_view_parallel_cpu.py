"""Host logic of the view-parallel step on CPU ranks (gloo, world size 2).

The rendering itself needs a GPU; here the backward is replaced by a
deterministic per-rank gradient so the sharding, the gradient all-reduce and
the failure path run as real separate processes over gloo.
"""

import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gaussian_splats_b200.view_parallel import all_reduce_gradients, shard_views, train_step


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_views_covers_each_view_once():
    for views in (1, 7, 8, 64):
        for world in (1, 2, 3, 4, 8):
            shards = [shard_views(views, world, r) for r in range(world)]
            flat = [v for s in shards for v in s]
            assert sorted(flat) == list(range(views))
            assert max(map(len, shards)) - min(map(len, shards)) <= 1
    with pytest.raises(ValueError):
        shard_views(8, 2, 2)


def test_single_process_step_keeps_local_gradients():
    params = [torch.ones(5, 3, requires_grad=True), torch.ones(5, 4, requires_grad=True)]
    cams, targets = [1.0, 2.0], [torch.zeros(()), torch.zeros(())]
    render = lambda s, cam: sum((p * cam).sum() for p in params)  # noqa: E731
    loss = train_step(None, cams, targets, params, render, lambda image, t: image - t)
    assert float(loss) == 3.0 * (15 + 20)
    assert torch.all(params[0].grad == 3.0) and torch.all(params[1].grad == 3.0)


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    params = [torch.zeros(100, 3, requires_grad=True), torch.zeros(100, 16, 3, requires_grad=True)]
    views = shard_views(8, world, rank)
    # Stand-in for rendering a view: the loss is (view index + 1) * sum(params).
    render = lambda s, v: sum((p * float(v + 1)).sum() for p in params)  # noqa: E731
    train_step(None, views, [0.0] * len(views), params, render, lambda image, t: image - t)
    results[rank] = (views, float(params[0].grad[0, 0]), float(params[1].grad[-1, -1, -1]))
    dist.destroy_process_group()


def test_all_reduce_sums_every_ranks_views():
    world = 2
    manager = mp.Manager()
    results = manager.dict()
    mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
    expected = float(sum(v + 1 for v in range(8)))  # every view counted once
    for rank in range(world):
        views, first, last = results[rank]
        assert first == expected and last == expected
    assert sorted(results[0][0] + results[1][0]) == list(range(8))


def _failing_worker(rank, world, port, results):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    params = [torch.zeros(10, requires_grad=True)]
    params[0].grad = torch.ones(10)
    if rank == 1:
        # This rank fails between steps: it leaves without joining the collective.
        results[rank] = "left"
        return
    start = time.time()
    try:
        all_reduce_gradients(params)
        results[rank] = "no error"
    except Exception as error:  # the survivor must see an error, not hang
        results[rank] = f"error after {time.time() - start:.1f}s: {type(error).__name__}"


def test_missing_rank_ends_collective_with_error():
    world = 2
    manager = mp.Manager()
    results = manager.dict()
    mp.spawn(_failing_worker, args=(world, _free_port(), results), nprocs=world, join=True)
    assert results[1] == "left"
    assert results[0].startswith("error after"), results[0]


def test_shared_flat_detection():
    from gaussian_splats_b200.view_parallel import _shared_flat

    flat = torch.arange(20, dtype=torch.float32)
    views = [flat[0:8].view(2, 4), flat[8:14].view(2, 3), flat[14:20].view(2, 3)]
    got = _shared_flat(views)
    assert got is not None and got.numel() == 20 and got.data_ptr() == flat.data_ptr()
    assert _shared_flat(views[:2]) is None  # does not cover the storage
    assert _shared_flat([torch.zeros(3), torch.zeros(4)]) is None  # separate storages
    assert _shared_flat([flat[0:10], flat[5:20]]) is None  # overlapping


def _flat_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    params = [torch.zeros(5, 4, requires_grad=True), torch.zeros(5, 3, requires_grad=True)]
    flat = torch.full((35,), float(rank + 1))
    params[0].grad, params[1].grad = flat[:20].view(5, 4), flat[20:].view(5, 3)
    all_reduce_gradients(params)
    results[rank] = (float(params[0].grad.sum()), float(params[1].grad.sum()),
                     params[0].grad.data_ptr() == flat.data_ptr())
    dist.destroy_process_group()


def test_flat_all_reduce_of_views():
    world = 2
    manager = mp.Manager()
    results = manager.dict()
    mp.spawn(_flat_worker, args=(world, _free_port(), results), nprocs=world, join=True)
    for rank in range(world):
        first, second, in_place = results[rank]
        assert first == 20 * 3.0 and second == 15 * 3.0 and in_place


def test_view_record_layout():
    import ctypes

    from gaussian_splats_b200 import native

    params = native.make_params(500.0, 510.0, 320.0, 240.0, 640, 480, 16, 0.999, 0.2, 100.0,
                                "gaussian", 0.95)
    R = torch.arange(9, dtype=torch.float32).reshape(3, 3)
    t = torch.tensor([1.5, -2.0, 3.25])
    words = native.view_record(params, R, t)
    assert words.dtype == torch.int32 and words.numel() == native.VIEW_RECORD_WORDS == 29
    assert ctypes.sizeof(native.Params) == 17 * 4
    back = native.Params.from_buffer_copy(words[:17].numpy().tobytes())
    assert (back.fx, back.width, back.tile_size, back.opacity_threshold) == \
        (params.fx, params.width, params.tile_size, params.opacity_threshold)
    assert torch.equal(words[17:].view(torch.float32), torch.cat((R.reshape(9), t)))


def test_screen_exchange_needs_one_view(monkeypatch):
    monkeypatch.setattr(dist, "is_initialized", lambda: True)
    monkeypatch.setattr(dist, "get_world_size", lambda group=None: 2)
    params = [torch.zeros(3, requires_grad=True)]
    with pytest.raises(ValueError, match="one view"):
        train_step(None, [1, 2], [0, 0], params, lambda s, c: params[0].sum(),
                   lambda image, t: image, screen_exchange=True)


def test_screen_exchange_is_seen_from_other_threads(monkeypatch):
    # autograd runs CUDA backward functions on its own device thread, so the
    # context set on the caller's thread must be visible there
    import threading

    from gaussian_splats_b200 import view_parallel

    monkeypatch.setattr(dist, "is_initialized", lambda: True)
    group = object()
    seen = []
    with view_parallel.screen_space_exchange(group):
        worker = threading.Thread(target=lambda: seen.append(view_parallel.active_exchange()))
        worker.start()
        worker.join()
    assert seen == [group]
    assert view_parallel.active_exchange() is None


def test_screen_exchange_choice():
    from gaussian_splats_b200.view_parallel import screen_exchange_pays

    assert [screen_exchange_pays(w, "p2p") for w in (1, 2, 4, 8)] == [False, True, True, False]
    assert [screen_exchange_pays(w, "p2p-shard") for w in (1, 2, 4, 8)] == [False, True, True,
                                                                           True]
    assert [screen_exchange_pays(w, "auto") for w in (1, 2, 4, 8)] == [False, True, True, True]


def test_collectives_are_counted_for_the_graph_guard(monkeypatch):
    from gaussian_splats_b200 import view_parallel

    monkeypatch.setattr(dist, "is_initialized", lambda: True)
    monkeypatch.setattr(dist, "get_world_size", lambda group=None: 2)
    monkeypatch.setattr(dist, "all_reduce", lambda *a, **k: None)
    before = view_parallel.COLLECTIVE_CALLS
    grads = [torch.zeros(3)]
    for g in grads:
        g.grad = torch.ones(3)
    all_reduce_gradients(grads)
    assert view_parallel.COLLECTIVE_CALLS == before + 1


def _arena_worker(rank, world, port, results):
    """Arena bookkeeping across a destroyed and re-created process group (the
    symmetric-memory arena itself is replaced by a stand-in: no GPU here)."""
    from gaussian_splats_b200 import view_parallel as vp

    made = []

    class FakeArena:
        def __init__(self, n, device, group, num_sh=None):
            made.append((n, group))

    vp.PeerArena = FakeArena
    device = torch.device("cpu")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    first = vp.peer_arena(10, device, None)
    assert vp.peer_arena(10, device, None) is first  # cached while the group lives
    dist.destroy_process_group()  # without release_arenas: the stale entry stays
    os.environ["MASTER_PORT"] = str(port + 1)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    second = vp.peer_arena(10, device, None)  # a new group gets a new arena
    released = vp.release_arenas(None)  # every group's arenas
    third = vp.peer_arena(10, device, None)
    assert vp.release_arenas(dist.group.WORLD) == 1
    dist.destroy_process_group()
    results[rank] = (second is not first, third is not second, released, len(made))


def test_arenas_are_rebuilt_for_a_recreated_group():
    world = 2
    manager = mp.Manager()
    results = manager.dict()
    port = _free_port()
    mp.spawn(_arena_worker, args=(world, port, results), nprocs=world, join=True)
    for rank in range(world):
        assert results[rank] == (True, True, 2, 3)
