"""Splat relocation on the GPU (gs_relocate behind gaussian_splats_b200.relocate)
against the reference-run fixture and the CPU oracle."""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

import oracle as O  # noqa: E402

from gaussian_splats_b200 import relocate as R  # noqa: E402
from gaussian_splats_b200.optim import FusedAdam  # noqa: E402
from gaussian_splats_b200.splats import GaussianSplat  # noqa: E402

from test_relocate_cpu import NAMES, check_state, replay_relocation  # noqa: E402

pytestmark = pytest.mark.gpu


def _fixture():
    return np.load(os.path.join(GOLDEN, "relocate.npz"))


def _splats(arrays: dict) -> GaussianSplat:
    return GaussianSplat.from_tensors(*(torch.tensor(arrays[k]).cuda() for k in NAMES))


def _host(splats: GaussianSplat) -> dict:
    return {k: getattr(splats, k).detach().cpu().numpy() for k in NAMES}


def _check_vs_oracle(got: dict, expected: dict) -> None:
    """Copies bit-exact; the renormalised values, each one double-precision
    result rounded to float on both sides, within one float ulp (CUDA's and
    the C library's double exp / log / pow differ in the last double bits)."""
    for name in NAMES:
        if name in ("scale", "opacity"):
            np.testing.assert_array_max_ulp(got[name], expected[name], maxulp=1)
        else:
            np.testing.assert_array_equal(got[name], expected[name], err_msg=name)


def test_copy_splats_matches_reference_and_oracle():
    d = _fixture()
    state = {k: d[f"copy_in_{k}"] for k in NAMES}
    splats = _splats(state)
    reset = R.copy_splats(splats, torch.tensor(d["copy_counts"]).cuda(),
                          torch.tensor(d["copy_outputs"]).cuda())
    got = _host(splats)
    check_state(got, {k: d[f"copy_out_{k}"] for k in NAMES})
    np.testing.assert_array_equal(reset.cpu().numpy(), d["copy_reset"])
    expected = O.relocate(state, d["copy_counts"], d["copy_outputs"])
    _check_vs_oracle(got, expected["state"])


@pytest.mark.parametrize("optimizer_class", [torch.optim.Adam, FusedAdam])
def test_relocate_splats_matches_reference(optimizer_class, monkeypatch):
    d = _fixture()
    splats = _splats({k: d[f"reloc_in_{k}"] for k in NAMES})
    params = [getattr(splats, k) for k in O.ADAM_NAMES]
    opt = optimizer_class([{"params": [p], "name": k, "lr": 1e-3}
                           for p, k in zip(params, O.ADAM_NAMES)], eps=1e-15)
    for k, p in zip(O.ADAM_NAMES, params):
        opt.state[p] = {"step": torch.tensor(1.0),
                        "exp_avg": torch.tensor(d[f"reloc_in_exp_avg_{k}"]).cuda(),
                        "exp_avg_sq": torch.tensor(d[f"reloc_in_exp_avg_sq_{k}"]).cuda()}
    draws = [torch.tensor(d["reloc_counts_dead"]).cuda(),
             torch.tensor(d["reloc_counts_densify"]).cuda()]
    monkeypatch.setattr(R, "sample_counts", lambda weights, count: draws.pop(0))
    R.relocate_splats(splats, opt, densification_factor=1.05)
    assert not draws
    got = _host(splats)
    check_state(got, {k: d[f"reloc_out_{k}"] for k in NAMES})
    for group in opt.param_groups:
        p = group["params"][0]
        assert p is getattr(splats, group["name"])
        for key in ("exp_avg", "exp_avg_sq"):
            np.testing.assert_array_equal(opt.state[p][key].cpu().numpy(),
                                          d[f"reloc_out_{key}_{group['name']}"])

    def oracle_step(state, counts, indices, base, m, v):
        out = O.relocate(state, counts, indices, base, exp_avg=m, exp_avg_sq=v)
        return out["state"], out["exp_avg"], out["exp_avg_sq"]

    expected, _, _ = replay_relocation(d, oracle_step)
    _check_vs_oracle(got, expected)
    # the optimizer keeps stepping on the grown parameters
    for p in opt.param_groups:
        p["params"][0].grad = torch.full_like(p["params"][0], 0.01)
    opt.step()
    assert all(torch.isfinite(getattr(splats, k)).all() for k in O.ADAM_NAMES)


def test_relocate_at_scale_matches_oracle(monkeypatch):
    """One million splats, SH degree 3, ~5 % dead, the reference's own random
    draws (torch.multinomial on the device); the oracle replays the same
    counts."""
    n = 1_000_000
    g = torch.Generator().manual_seed(8)
    state = {"mean": torch.randn(n, 3, generator=g), "rotation": torch.randn(n, 4, generator=g),
             "scale": torch.randn(n, 3, generator=g) * 0.5 - 4.0,
             "opacity": torch.randn(n, 1, generator=g) * 2.0 - 1.5,
             "color": torch.randn(n, 16, 3, generator=g) * 0.3,
             "normals": torch.randn(n, 3, generator=g)}
    splats = GaussianSplat.from_tensors(*(state[k].cuda() for k in NAMES))
    drawn = []
    sample = R.sample_counts

    def recording(weights, count):
        out = sample(weights, count)
        drawn.append(out.cpu().numpy())
        return out

    monkeypatch.setattr(R, "sample_counts", recording)
    torch.manual_seed(0)
    R.relocate_splats(splats, None, densification_factor=1.02)
    got = _host(splats)
    host = {k: v.numpy() for k, v in state.items()}
    # dead rows as relocate_splats finds them (the device's sigmoid)
    dead = (torch.sigmoid(state["opacity"].cuda()).squeeze(-1) < 0.005).nonzero().squeeze(-1)
    dead = dead.cpu().numpy()
    assert len(drawn) == 2 and drawn[0].sum() == len(dead) > 10_000
    first = O.relocate(host, drawn[0], dead)["state"]
    diff = int(drawn[1].sum())
    grown = {k: np.concatenate((v, np.zeros((diff,) + v.shape[1:], v.dtype)))
             for k, v in first.items()}
    expected = O.relocate(grown, drawn[1], None, n)
    assert expected["error"] == 0 and len(got["mean"]) == n + diff == int(1.02 * n)
    _check_vs_oracle(got, expected["state"])


def test_bad_counts_and_rows_are_reported_not_written():
    d = _fixture()
    state = {k: d[f"copy_in_{k}"] for k in NAMES}
    counts = torch.tensor(d["copy_counts"]).cuda()
    outputs = torch.tensor(d["copy_outputs"]).cuda()
    splats = _splats(state)
    # one more copy than output rows: the extra slot is skipped and reported
    bad = counts.clone()
    bad[int(torch.nonzero(counts)[0])] += 1
    workspace = R._relocate(splats, bad, outputs, 0, len(outputs), (None, None))
    with pytest.raises(RuntimeError, match="gs_relocate"):
        R._check(workspace)
    # an output row outside the set: that slot is skipped and reported
    splats = _splats(state)
    rows = outputs.clone()
    rows[5] = len(counts) + 7
    workspace = R._relocate(splats, counts, rows, 0, len(rows), (None, None))
    with pytest.raises(RuntimeError, match="gs_relocate"):
        R._check(workspace)
    expected = O.relocate(state, d["copy_counts"], rows.cpu().numpy())
    assert expected["error"] == 4
    _check_vs_oracle(_host(splats), expected["state"])
    with pytest.raises(RuntimeError, match="add up"):
        R.copy_splats(_splats(state), bad, outputs)
