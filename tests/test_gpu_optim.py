"""Fused optimizer step (gs_adam_step / FusedAdam) on the GPU.

Against the CPU oracle, which evaluates the same float32 operations in the
same order, the step is bit-identical (parameters and both moments, with and
without the position noise, with skipped groups and odd sizes). Against
torch.optim.Adam on the GPU, the reference-run fixture and the reference's
noise formula it agrees to float32 rounding (rtol 1e-5, atol 1e-6).
"""

import ctypes
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

from gaussian_splats_b200 import native
from gaussian_splats_b200.optim import GROUP_NAMES, FusedAdam

pytestmark = pytest.mark.gpu

SHAPES = {"mean": 3, "rotation": 4, "scale": 3, "opacity": 1}


def _random_splat(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    return {"mean": torch.randn(n, 3, generator=g),
            "rotation": torch.randn(n, 4, generator=g),
            "scale": torch.randn(n, 3, generator=g) * 0.5 - 4.0,
            "opacity": torch.randn(n, 1, generator=g) * 3.0 - 4.0,
            "color": torch.randn(n, k, 3, generator=g) * 0.3}


def _optimizer(params, lrs, cls):
    groups = [{"params": [params[name]], "name": name, "lr": lr}
              for name, lr in zip(GROUP_NAMES, lrs)]
    return cls(groups, eps=1e-15)


@pytest.mark.parametrize("n,k", [(1, 1), (257, 16), (1000, 4), (4099, 9)])
def test_bit_exact_vs_oracle(oracle, n, k):
    host = _random_splat(n, k, seed=n + k)
    params = {name: t.cuda().requires_grad_() for name, t in host.items()}
    lrs = [5e-4, 1e-3, 5e-3, 5e-2, 2.5e-3]
    opt = _optimizer(params, lrs, FusedAdam)
    p = {name: t.numpy() for name, t in host.items()}
    m = {name: np.zeros_like(x) for name, x in p.items()}
    v = {name: np.zeros_like(x) for name, x in p.items()}
    steps = [0] * 5
    g = torch.Generator().manual_seed(7)
    for it in range(4):
        grads = {}
        for i, name in enumerate(GROUP_NAMES):
            skip = it == 1 and name in ("scale", "color")
            grad = None if skip else torch.randn(host[name].shape, generator=g) * 10.0 ** -it
            params[name].grad = None if grad is None else grad.cuda()
            grads[name] = None if grad is None else grad.numpy()
            steps[i] += 0 if skip else 1
        noise = (5e5, 5e-4) if it % 2 else None
        if noise:
            torch.cuda.manual_seed(100 + it)
            randn = torch.randn(n, 3, device="cuda").cpu().numpy()
            torch.cuda.manual_seed(100 + it)
        opt.step(noise=noise)
        hyper = oracle.adam_scalars(steps, lrs, eps=1e-15, noise_lr=noise[0] if noise else 0.0,
                                    position_lr=noise[1] if noise else 0.0)
        out = oracle.adam_step(p, grads, m, v, hyper, randn=randn if noise else None)
        p, m, v = out["params"], out["exp_avg"], out["exp_avg_sq"]
    for name in GROUP_NAMES:
        t = params[name]
        np.testing.assert_array_equal(t.detach().cpu().numpy(), p[name], err_msg=name)
        np.testing.assert_array_equal(opt.state[t]["exp_avg"].cpu().numpy(), m[name])
        np.testing.assert_array_equal(opt.state[t]["exp_avg_sq"].cpu().numpy(), v[name])


def test_matches_torch_adam_on_gpu():
    host = _random_splat(3001, 16, seed=5)
    lrs = [5e-4, 1e-3, 5e-3, 5e-2, 2.5e-3]
    ours = {name: t.cuda().requires_grad_() for name, t in host.items()}
    theirs = {name: t.cuda().requires_grad_() for name, t in host.items()}
    fused, plain = _optimizer(ours, lrs, FusedAdam), _optimizer(theirs, lrs, torch.optim.Adam)
    g = torch.Generator().manual_seed(8)
    for it in range(5):
        for name in GROUP_NAMES:
            grad = (torch.randn(host[name].shape, generator=g) * 0.1).cuda()
            ours[name].grad, theirs[name].grad = grad.clone(), grad.clone()
        fused.step()
        plain.step()
    for name in GROUP_NAMES:
        torch.testing.assert_close(ours[name], theirs[name], rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(fused.state[ours[name]]["exp_avg_sq"],
                                   plain.state[theirs[name]]["exp_avg_sq"], rtol=1e-5,
                                   atol=1e-12)


def _noise_splats_torch(params, noise_lr, position_lr):
    """The reference's noise_splats (training/utils.py:50-62), restated in torch."""
    q = torch.nn.functional.normalize(params["rotation"], dim=-1)
    w, x, y, z = q.unbind(-1)
    r = torch.stack((1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
                     2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
                     2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)),
                    -1).reshape(-1, 3, 3)
    factor = r * params["scale"].exp()[:, None, :]
    covariance = factor @ factor.transpose(-1, -2)
    gate = torch.sigmoid(100 * (1 - params["opacity"].sigmoid() - 0.995))
    noise = torch.randn_like(params["mean"]) * gate * noise_lr * position_lr
    params["mean"].add_((covariance @ noise[..., None]).squeeze(-1))


def test_noise_matches_reference_formula():
    host = _random_splat(2048, 4, seed=9)
    lrs = [5e-4, 1e-3, 5e-3, 5e-2, 2.5e-3]
    ours = {name: t.cuda().requires_grad_() for name, t in host.items()}
    theirs = {name: t.cuda().requires_grad_() for name, t in host.items()}
    fused, plain = _optimizer(ours, lrs, FusedAdam), _optimizer(theirs, lrs, torch.optim.Adam)
    for name in GROUP_NAMES:
        grad = torch.full_like(ours[name], 0.01)
        ours[name].grad, theirs[name].grad = grad.clone(), grad.clone()
    torch.cuda.manual_seed(77)
    fused.step(noise=(5e5, 5e-4))
    torch.cuda.manual_seed(77)
    plain.step()
    with torch.no_grad():
        _noise_splats_torch(theirs, 5e5, 5e-4)
    moved = (theirs["mean"] - host["mean"].cuda()).abs().max()
    assert moved > 1e-3
    torch.testing.assert_close(ours["mean"], theirs["mean"], rtol=1e-5, atol=1e-6)


def test_reference_fixture_on_gpu():
    d = np.load(os.path.join(GOLDEN, "adam_noise.npz"))
    lrs = [float(x) for x in d["in_lrs"]]
    names = GROUP_NAMES
    p = {k: torch.from_numpy(d[f"in_{k}"]).cuda() for k in names}
    m = {k: torch.zeros_like(t) for k, t in p.items()}
    v = {k: torch.zeros_like(t) for k, t in p.items()}
    lib = native.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    arrays = lambda ts: native.SplatArrays(*(t.data_ptr() if t is not None else None  # noqa: E731
                                             for t in ts))
    n, k = p["mean"].shape[0], p["color"].shape[1]
    for step in range(3):
        grads = [torch.from_numpy(d[f"in_grad{step}_{name}"]).cuda() for name in names]
        hyper = native.adam_params([step + 1] * 5, lrs, (0.9, 0.999), 1e-15)
        native.check(lib.gs_adam_step(n, k, ctypes.byref(arrays([p[x] for x in names])),
                                      ctypes.byref(arrays(grads)),
                                      ctypes.byref(arrays([m[x] for x in names])),
                                      ctypes.byref(arrays([v[x] for x in names])),
                                      ctypes.byref(hyper), None, stream), "gs_adam_step")
    for name in names:
        np.testing.assert_allclose(p[name].cpu().numpy(), d[f"adam_{name}"], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(m[name].cpu().numpy(), d[f"exp_avg_{name}"], rtol=1e-4,
                                   atol=1e-8)
    randn = torch.from_numpy(d["in_randn"]).cuda()
    noise_lr, position_lr = (float(x) for x in d["in_noise"])
    hyper = native.adam_params([4] * 5, lrs, (0.9, 0.999), 1e-15, noise_lr, position_lr)
    none = native.SplatArrays()
    native.check(lib.gs_adam_step(n, k, ctypes.byref(arrays([p[x] for x in names])),
                                  ctypes.byref(none), ctypes.byref(arrays([m[x] for x in names])),
                                  ctypes.byref(arrays([v[x] for x in names])), ctypes.byref(hyper),
                                  ctypes.c_void_p(randn.data_ptr()), stream), "gs_adam_step")
    np.testing.assert_allclose(p["mean"].cpu().numpy(), d["noised_mean"], rtol=1e-5, atol=1e-6)


def test_state_edits_like_relocation(oracle):
    """relocate_splats zeroes the moments of relocated rows and grows every
    tensor when densifying (training/utils.py:187-210); FusedAdam keeps
    working on the edited state."""
    host = _random_splat(500, 16, seed=12)
    lrs = [5e-4, 1e-3, 5e-3, 5e-2, 2.5e-3]
    params = {name: t.cuda().requires_grad_() for name, t in host.items()}
    opt = _optimizer(params, lrs, FusedAdam)
    for name in GROUP_NAMES:
        params[name].grad = torch.full_like(params[name], 0.05)
    opt.step()
    rows = torch.tensor([3, 17, 499], device="cuda")
    for state in opt.state.values():
        for key in ("exp_avg", "exp_avg_sq"):
            state[key][rows] = 0
    grown = {}
    with torch.no_grad():
        for group in opt.param_groups:
            old = group["params"][0]
            new = torch.cat((old, old[:8])).requires_grad_()
            state = opt.state.pop(old)
            for key in ("exp_avg", "exp_avg_sq"):
                state[key] = torch.cat((state[key], torch.zeros_like(new[-8:])))
            opt.state[new] = state
            group["params"][0] = new
            grown[group["name"]] = new
    before = {name: t.detach().cpu().numpy() for name, t in grown.items()}
    m = {name: opt.state[t]["exp_avg"].cpu().numpy() for name, t in grown.items()}
    v = {name: opt.state[t]["exp_avg_sq"].cpu().numpy() for name, t in grown.items()}
    grads = {}
    for name, t in grown.items():
        t.grad = torch.full_like(t, -0.02)
        grads[name] = t.grad.cpu().numpy()
    opt.step()
    out = oracle.adam_step(before, grads, m, v, oracle.adam_scalars(2, lrs, eps=1e-15))
    for name, t in grown.items():
        np.testing.assert_array_equal(t.detach().cpu().numpy(), out["params"][name])
