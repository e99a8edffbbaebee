"""One rank of the screen-space exchange check, run under torch.distributed.run
by tests/test_gpu_views_backward.py when two or more GPUs are present.

Each rank renders its own camera of one shared scene; ``train_step`` with the
screen-space exchange (all-gather of screen-space gradients, one projection
backward over every rank's view) must give the gradients of ``train_step``
with the parameter-gradient all-reduce, on every rank -- with the screen-space
gradients all-gathered by NCCL, copied whole from peer memory, and sharded
(each rank computing the summed projection backward of its own shard of
Gaussians and copying the others' finished shards) -- the two peer-memory
forms also replayed from a CUDA graph, which they allow: they issue no
collective.
"""

import datetime
import math
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from gaussian_splats_b200 import scenes  # noqa: E402
from gaussian_splats_b200 import view_parallel as VP  # noqa: E402
from gaussian_splats_b200.graphs import CapturedStep  # noqa: E402
from gaussian_splats_b200.rasterize import rasterize_outputs  # noqa: E402
from gaussian_splats_b200.splats import GaussianSplat  # noqa: E402
from gaussian_splats_b200.view_parallel import train_step  # noqa: E402


def main():
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(rank)
    try:
        g = torch.Generator().manual_seed(11)
        tensors = scenes.random_gaussians(g, 60_000, means=("normal", 0.0, 1.0),
                                          log_scale=(-4.5, 0.7), opacity_logit=(0.0, 1.5),
                                          sh_degree=3)
        splats = GaussianSplat.from_tensors(*(t.cuda() for t in tensors))
        params = [splats.mean, splats.rotation, splats.scale, splats.opacity, splats.color]
        for p in params:
            p.requires_grad_(True)
        angle = 2 * math.pi * rank / world
        camera = scenes.look_at_camera((4 * math.cos(angle), 0.7, 4 * math.sin(angle)),
                                       fovy_degrees=50.0, width=320, height=240)
        target = torch.rand(240, 320, 3, generator=torch.Generator().manual_seed(rank)).cuda()

        def render(s, c):
            return rasterize_outputs(s, c, 16)[0]

        def loss_fn(image, t):
            return (image[:240, :320] - t).abs().mean()

        # gradients summed by all-reducing them, and inside the backward by
        # the screen-space exchange over NCCL and over peer memory
        results = {}
        exchanges = ("nccl", "p2p", "p2p-shard")
        for mode in ("all-reduce",) + exchanges:
            VP.EXCHANGE_TRANSPORT = "p2p" if mode == "all-reduce" else mode
            train_step(splats, [camera], [target], params, render, loss_fn,
                       screen_exchange=mode != "all-reduce")
            results[mode] = [p.grad.clone() for p in params]
        names = ("mean", "rotation", "scale", "opacity", "color")
        for mode in exchanges:
            for name, a, b in zip(names, results["all-reduce"], results[mode]):
                # compositing backward's float atomics add in scheduling order,
                # and the paths sum the views in different orders: the
                # absolute tolerance is on the scale of the gradient tensor
                torch.testing.assert_close(b, a, rtol=1e-4, atol=1e-4 * float(a.abs().max()),
                                           msg=lambda m: f"{mode} {name}: {m}")
                assert torch.count_nonzero(a) > 0, name
            for grad in results[mode]:  # every rank holds the same summed gradients
                ref = grad.clone()
                dist.broadcast(ref, 0)
                assert torch.equal(ref, grad), mode
        # the peer-memory steps replayed from a CUDA graph (they issue no collective)
        for mode in ("p2p", "p2p-shard"):
            VP.EXCHANGE_TRANSPORT = mode
            step = CapturedStep(lambda: train_step(splats, [camera], [target], params, render,
                                                   loss_fn, screen_exchange=True))
            for _ in range(3):
                step()
            assert step.check()
            VP.check_exchange()
            for name, a, p in zip(names, results[mode], params):
                torch.testing.assert_close(p.grad, a, rtol=1e-4,
                                           atol=1e-4 * float(a.abs().max()),
                                           msg=lambda m: f"graph {mode} {name}: {m}")
            del step
        # the other ranks' views really were added in: the summed gradient
        # differs from this rank's own view alone
        for p in params:
            p.grad = None
        loss_fn(render(splats, camera), target).backward()
        own = params[0].grad
        assert (own - results["p2p"][0]).abs().max() > 10 * own.abs().max() * 1e-4
        dist.barrier()
        if rank == 0:
            print(f"exchange ok at world {world}", flush=True)
    finally:
        VP.release_arenas()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
