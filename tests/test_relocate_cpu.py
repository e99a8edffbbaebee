"""Splat relocation on CPU: the oracle's restatement of copy_splats /
normalize_copies / the moment reset against the reference-run fixture
(tests/golden/relocate.npz, made by tests/golden/make_goldens.py), its error
bits, and the host logic of gaussian_splats_b200.relocate."""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

import oracle as O  # noqa: E402

from gaussian_splats_b200 import relocate as R  # noqa: E402
from gaussian_splats_b200.splats import GaussianSplat  # noqa: E402

NAMES = O.ADAM_NAMES + ("normals",)
# The reference renormalises in float32; the oracle in double, rounded once.
# Their difference is the reference's rounding: largest for the log scale of
# a parent with 51 copies, whose alternating binomial series cancels.
LOG_SCALE_ATOL = 3e-5
OPACITY_ATOL = 2e-6


def _fixture():
    return np.load(os.path.join(GOLDEN, "relocate.npz"))


def check_state(got: dict, expected: dict) -> None:
    """Copies exact, renormalised opacity / log scale within the tolerance."""
    for name in NAMES:
        a, b = np.asarray(got[name]), np.asarray(expected[name])
        if name == "scale":
            np.testing.assert_allclose(a, b, rtol=0, atol=LOG_SCALE_ATOL, err_msg=name)
        elif name == "opacity":
            np.testing.assert_allclose(a, b, rtol=0, atol=OPACITY_ATOL, err_msg=name)
        else:
            np.testing.assert_array_equal(a, b, err_msg=name)


def replay_relocation(d, relocate):
    """The relocate_splats flow (training/utils.py:147-210) with the fixture's
    recorded draws; ``relocate(state, counts, indices, base, m, v)`` returns
    (state, m, v)."""
    state = {k: d[f"reloc_in_{k}"] for k in NAMES}
    m = {k: d[f"reloc_in_exp_avg_{k}"] for k in O.ADAM_NAMES}
    v = {k: d[f"reloc_in_exp_avg_sq_{k}"] for k in O.ADAM_NAMES}
    opacity = torch.sigmoid(torch.from_numpy(state["opacity"])).squeeze(-1)
    dead = (opacity < 0.005).nonzero().squeeze(-1).numpy()
    state, m, v = relocate(state, d["reloc_counts_dead"], dead, 0, m, v)
    n, diff = len(state["mean"]), int(d["reloc_counts_densify"].sum())

    def grow(a):
        return np.concatenate((a, np.zeros((diff,) + a.shape[1:], a.dtype)))

    state = {k: grow(a) for k, a in state.items()}
    m = {k: grow(a) for k, a in m.items()}
    v = {k: grow(a) for k, a in v.items()}
    return relocate(state, d["reloc_counts_densify"], None, n, m, v)


def _oracle_relocate(state, counts, indices, base, m, v):
    out = O.relocate(state, counts, indices, base, exp_avg=m, exp_avg_sq=v)
    assert out["error"] == 0
    return out["state"], out["exp_avg"], out["exp_avg_sq"]


def test_oracle_copy_splats_matches_reference():
    d = _fixture()
    state = {k: d[f"copy_in_{k}"] for k in NAMES}
    assert d["copy_counts"].max() > 51  # normalize_copies' clamp is exercised
    out = O.relocate(state, d["copy_counts"], d["copy_outputs"])
    assert out["error"] == 0
    check_state(out["state"], {k: d[f"copy_out_{k}"] for k in NAMES})
    # rows outside parents and outputs are untouched
    touched = np.zeros(len(d["copy_counts"]), bool)
    touched[d["copy_reset"]] = True
    for k in NAMES:
        np.testing.assert_array_equal(out["state"][k][~touched], state[k][~touched])


def test_oracle_relocate_splats_matches_reference():
    d = _fixture()
    state, m, v = replay_relocation(d, _oracle_relocate)
    check_state(state, {k: d[f"reloc_out_{k}"] for k in NAMES})
    for k in O.ADAM_NAMES:
        np.testing.assert_array_equal(m[k], d[f"reloc_out_exp_avg_{k}"])
        np.testing.assert_array_equal(v[k], d[f"reloc_out_exp_avg_sq_{k}"])
    assert len(state["mean"]) == len(d["reloc_out_mean"]) > len(d["reloc_in_mean"])


def test_oracle_error_bits():
    d = _fixture()
    state = {k: d[f"copy_in_{k}"] for k in NAMES}
    counts = d["copy_counts"].copy()
    outputs = d["copy_outputs"]
    assert O.relocate(state, counts[:-1] if counts[-1] == 0 else counts, outputs)["error"] == 0
    bad = counts.copy()
    bad[np.flatnonzero(counts)[0]] += 1  # one copy more than output rows
    assert O.relocate(state, bad, outputs)["error"] & 2
    negative = counts.copy()
    negative[np.flatnonzero(counts == 0)[0]] = -1
    assert O.relocate(state, negative, outputs)["error"] & 1
    out_of_range = outputs.copy()
    out_of_range[3] = len(counts)
    result = O.relocate(state, counts, out_of_range)
    assert result["error"] == 4
    assert result["state"]["mean"].shape == state["mean"].shape


def test_relocate_has_no_cpu_path():
    splats = GaussianSplat(64, sh_degree=1)
    with torch.no_grad():
        splats.opacity[:8] = -8.0  # dead rows
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        R.relocate_splats(splats)


def test_relocate_rejects_other_optimizers_before_editing():
    splats = GaussianSplat(32, sh_degree=1)
    with torch.no_grad():
        splats.opacity[:4] = -8.0
    before = splats.opacity.detach().clone()
    sgd = torch.optim.SGD(splats.parameters(), lr=0.1)
    with pytest.raises(TypeError, match="Adam, AdamW, or None"):
        R.relocate_splats(splats, sgd, densification_factor=1.5)
    assert torch.equal(splats.opacity.detach(), before) and len(splats.mean) == 32


def test_sample_counts_and_append_like_reference():
    g = torch.Generator().manual_seed(0)
    weights = torch.rand(50, generator=g)
    torch.manual_seed(3)
    counts = R.sample_counts(weights, 40)
    torch.manual_seed(3)
    expected = torch.bincount(torch.multinomial(weights, 40, replacement=True), minlength=50)
    assert torch.equal(counts, expected) and counts.dtype == torch.int64
    splats = GaussianSplat(10, sh_degree=2)
    grown = R.append_empty_splats(splats, 5)
    assert grown.sh_degree == 2
    for name in NAMES:
        value = getattr(grown, name)
        assert isinstance(value, torch.nn.Parameter) and len(value) == 15
        assert torch.equal(value[:10], getattr(splats, name).detach())
        assert torch.count_nonzero(value[10:]) == 0
