"""Optimizer step (Adam + position noise) on CPU: the oracle against the
reference-run fixture and against torch.optim.Adam, and the host logic of
FusedAdam (group checks, step folding, no CPU path)."""

import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402

from gaussian_splats_b200 import native  # noqa: E402
from gaussian_splats_b200.optim import GROUP_NAMES, FusedAdam  # noqa: E402

GOLDEN = os.path.join(ROOT, "tests", "golden", "adam_noise.npz")


def _replay(d, noise=True):
    lrs = list(d["in_lrs"])
    p = {k: d[f"in_{k}"] for k in O.ADAM_NAMES}
    m = {k: np.zeros_like(v) for k, v in p.items()}
    v = {k: np.zeros_like(x) for k, x in p.items()}
    for step in range(3):
        out = O.adam_step(p, {k: d[f"in_grad{step}_{k}"] for k in O.ADAM_NAMES}, m, v,
                          O.adam_scalars(step + 1, lrs))
        p, m, v = out["params"], out["exp_avg"], out["exp_avg_sq"]
    adam = {k: x.copy() for k, x in p.items()}
    if noise:
        noise_lr, position_lr = d["in_noise"]
        out = O.adam_step(p, {k: None for k in O.ADAM_NAMES}, m, v,
                          O.adam_scalars(4, lrs, noise_lr=noise_lr, position_lr=position_lr),
                          randn=d["in_randn"])
        p = out["params"]
    return adam, m, v, p


def test_oracle_matches_reference_adam_and_noise():
    d = np.load(GOLDEN)
    adam, m, v, noised = _replay(d)
    for k in O.ADAM_NAMES:
        np.testing.assert_allclose(adam[k], d[f"adam_{k}"], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(m[k], d[f"exp_avg_{k}"], rtol=1e-4, atol=1e-8)
        np.testing.assert_allclose(v[k], d[f"exp_avg_sq_{k}"], rtol=1e-5, atol=1e-10)
    # noise_splats moved the means by up to ~0.6; the oracle reproduces the move
    shift = d["noised_mean"] - d["adam_mean"]
    assert np.abs(shift).max() > 0.1
    np.testing.assert_allclose(noised["mean"], d["noised_mean"], rtol=1e-5, atol=1e-6)
    for k in O.ADAM_NAMES[1:]:
        np.testing.assert_array_equal(noised[k], adam[k])  # noise touches only the means


def test_oracle_matches_torch_adam_with_skipped_groups():
    rng = np.random.default_rng(3)
    shapes = [(33, 3), (33, 4), (33, 3), (33, 1), (33, 4, 3)]
    p0 = {k: rng.standard_normal(s).astype(np.float32) for k, s in zip(O.ADAM_NAMES, shapes)}
    lrs = [1e-3, 2e-3, 3e-3, 4e-3, 5e-3]
    tensors = [torch.tensor(p0[k], requires_grad=True) for k in O.ADAM_NAMES]
    opt = torch.optim.Adam([{"params": [t], "lr": lr} for t, lr in zip(tensors, lrs)],
                           eps=1e-15)
    p, m, v = p0, {k: np.zeros_like(x) for k, x in p0.items()}, \
        {k: np.zeros_like(x) for k, x in p0.items()}
    steps = [0] * 5
    for it in range(4):
        grads = {}
        for i, (k, t) in enumerate(zip(O.ADAM_NAMES, tensors)):
            skip = (it == 0 and k == "opacity") or (it == 2 and k == "color")
            grads[k] = None if skip else (rng.standard_normal(t.shape) * 0.1).astype(np.float32)
            t.grad = None if skip else torch.tensor(grads[k])
            steps[i] += 0 if skip else 1
        opt.step()
        out = O.adam_step(p, grads, m, v, O.adam_scalars([max(1, s) for s in steps], lrs))
        p, m, v = out["params"], out["exp_avg"], out["exp_avg_sq"]
    for k, t in zip(O.ADAM_NAMES, tensors):
        np.testing.assert_allclose(p[k], t.detach().numpy(), rtol=1e-6, atol=1e-7)


def test_step_folding_matches_oracle():
    a = native.adam_params([1, 2, 3, 4, 5], [1e-3, 2e-3, 3e-3, 4e-3, 5e-3], (0.9, 0.999), 1e-15,
                           5e5, 1.6e-4)
    for k, step in enumerate([1, 2, 3, 4, 5]):
        b = O.adam_scalars(step, [1e-3, 2e-3, 3e-3, 4e-3, 5e-3], eps=1e-15, noise_lr=5e5,
                           position_lr=1.6e-4)
        assert a.neg_step_size[k] == b.neg_step_size[k]
        assert a.bias2_sqrt[k] == b.bias2_sqrt[k]
    assert (a.lerp_weight, a.beta2, a.sq_weight, a.eps, a.noise_lr, a.position_lr) == \
        (b.lerp_weight, b.beta2, b.sq_weight, b.eps, b.noise_lr, b.position_lr)


def _groups(n=8, k=4):
    tensors = [torch.zeros(n, 3), torch.zeros(n, 4), torch.zeros(n, 3), torch.zeros(n, 1),
               torch.zeros(n, k, 3)]
    return [{"params": [t.requires_grad_()], "name": name, "lr": 1e-3}
            for t, name in zip(tensors, GROUP_NAMES)]


def test_fused_adam_checks_its_groups():
    FusedAdam(_groups(), eps=1e-15)
    with pytest.raises(ValueError):
        FusedAdam(_groups()[:4])
    bad = _groups()
    bad[0]["name"] = "position"
    with pytest.raises(ValueError):
        FusedAdam(bad)
    with pytest.raises(ValueError):
        FusedAdam(_groups(), weight_decay=0.1)


def test_fused_adam_has_no_cpu_path():
    opt = FusedAdam(_groups(), eps=1e-15)
    for group in opt.param_groups:
        group["params"][0].grad = torch.ones_like(group["params"][0])
    with pytest.raises(RuntimeError, match="no CPU path"):
        opt.step()
