"""Projection backward summed over views (gs_project_bwd_views) and the
screen-space gradient exchange of view-parallel training, on one GPU."""

import ctypes
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist

from gaussian_splats_b200 import native, scenes
from gaussian_splats_b200.rasterize import rasterize_outputs
from gaussian_splats_b200.splats import GaussianSplat
from gaussian_splats_b200.view_parallel import screen_space_exchange

pytestmark = pytest.mark.gpu


def _scene(k_degree=3, n=20_000, seed=3):
    g = torch.Generator().manual_seed(seed)
    tensors = scenes.random_gaussians(g, n, means=("normal", 0.0, 1.0), log_scale=(-4.0, 0.7),
                                      opacity_logit=(0.0, 1.5), sh_degree=k_degree)
    splats = GaussianSplat.from_tensors(*(t.cuda() for t in tensors))
    for p in (splats.mean, splats.rotation, splats.scale, splats.opacity, splats.color):
        p.requires_grad_(True)
    return splats


def _cameras(views):
    return [scenes.look_at_camera((4 * math.cos(2 * math.pi * v / views), 0.5,
                                   4 * math.sin(2 * math.pi * v / views)),
                                  fovy_degrees=55.0, width=128, height=96) for v in range(views)]


def _screen_gradients(splats, camera, seed):
    """One view's screen-space gradient (gs_composite_bwd) and forward outputs."""
    lib = native.lib()
    out = rasterize_outputs(splats, camera, 16)
    image, final_t, n_contrib, pm, conic, rgb, op, ids, ranges, counts = (o.detach() for o in out)
    g = torch.Generator(device="cuda").manual_seed(seed)
    grad_image = torch.randn(image.shape, device="cuda", generator=g)
    fx, fy = camera.focal_length
    cx, cy = camera.principal_point
    w, h = camera.image_size
    params = native.make_params(fx, fy, cx, cy, w, h, 16, 0.999, 0.2, 100.0, "gaussian", 0.95)
    n = pm.shape[0]
    gp = torch.empty((n, 9), device="cuda")
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    records = torch.empty((n, 16), device="cuda")
    native.check(lib.gs_pack_records(n, P(pm), P(conic), P(rgb), P(op), ctypes.byref(params),
                                     P(records), stream), "pack_records")
    native.check(lib.gs_composite_bwd(n, P(records), P(ids), P(ranges), P(grad_image),
                                      P(final_t), P(n_contrib), ctypes.byref(params), P(gp),
                                      None, stream), "composite_bwd")
    return params, conic, counts, gp, grad_image


@pytest.mark.parametrize("views,k", [(1, 3), (3, 3), (5, 1), (2, 4)])
def test_views_backward_is_the_sum_of_single_views(views, k):
    splats = _scene(k_degree=k)
    lib = native.lib()
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    tensors = [t.detach() for t in (splats.mean, splats.rotation, splats.scale, splats.opacity,
                                    splats.color)]
    n, num_sh = tensors[0].shape[0], tensors[4].shape[1]
    total = [torch.zeros_like(t) for t in tensors]
    gps, counts_all, records = [], [], []
    for v, camera in enumerate(_cameras(views)):
        params, conic, counts, gp, _ = _screen_gradients(splats, camera, seed=v)
        single = [torch.empty_like(t) for t in tensors]
        R, t = camera.rotation_matrix.cuda(), camera.translation.cuda()
        native.check(lib.gs_project_bwd(n, num_sh, *(P(x) for x in tensors), P(R), P(t),
                                        P(conic), P(gp), P(counts), ctypes.byref(params),
                                        *(P(x) for x in single), stream), "project_bwd")
        total = [a + b for a, b in zip(total, single)]  # the kernel's order: views in turn
        gps.append(gp)
        counts_all.append(counts)
        records.append(native.view_record(params, camera.rotation_matrix, camera.translation))
    gp_all, counts_all = torch.stack(gps), torch.stack(counts_all)
    views_dev = torch.stack(records).cuda()
    summed = [torch.empty_like(t) for t in tensors]
    native.check(lib.gs_project_bwd_views(n, num_sh, views, *(P(x) for x in tensors),
                                          P(views_dev), P(gp_all), P(counts_all),
                                          *(P(x) for x in summed), stream), "project_bwd_views")
    for a, b in zip(summed, total):
        assert torch.equal(a, b)
    assert any(torch.count_nonzero(x) > 0 for x in summed)


def test_exchange_plumbing_on_one_rank():
    """A one-rank NCCL group: the exchange path (all-gather of screen-space
    gradients, counts and view records; summed backward over the gathered
    views) must give the ordinary backward's gradients. The two backward
    passes each run compositing backward, whose float atomics add in
    scheduling order, so they agree to rounding, not bit for bit (the summed
    backward itself is bit-exact: test above); a component that is a sum with
    cancellation can differ by that rounding relative to the tensor's scale."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    try:
        camera = _cameras(1)[0]
        grads = []
        for exchange in (False, True):
            splats = _scene()
            params = [splats.mean, splats.rotation, splats.scale, splats.opacity, splats.color]
            image = rasterize_outputs(splats, camera, 16)[0]
            g = torch.Generator(device="cuda").manual_seed(5)
            weights = torch.randn(image.shape, device="cuda", generator=g)
            if exchange:
                with screen_space_exchange():
                    (image * weights).sum().backward()
            else:
                (image * weights).sum().backward()
            grads.append([p.grad.clone() for p in params])
        for a, b in zip(*grads):
            # summation order noise of the atomics, on sums with cancellation:
            # absolute, on the scale of the gradient tensor
            torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-4 * float(b.abs().max()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_exchange_matches_all_reduce_on_several_gpus():
    """One NCCL rank per GPU (up to eight), one camera each: train_step with
    every screen-space exchange gives the all-reduce path's gradients on every
    rank."""
    import subprocess
    import sys

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    worker = os.path.join(os.path.dirname(os.path.abspath(__file__)), "views_exchange_worker.py")
    world = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    run = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                          f"--nproc-per-node={world}", "--master-addr=127.0.0.1",
                          f"--master-port={port}", worker],
                         env=env, capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-3000:]
    assert f"exchange ok at world {world}" in run.stdout
