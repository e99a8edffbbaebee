"""Accuracy of the deterministic exp / log that fix the operator's numerics.

Both the CUDA kernels and the oracle evaluate these algorithms; the GPU test
``test_gpu_detmath.py`` checks the two copies agree bit for bit. Here the
oracle copy is checked against float64 numpy: at most 1 ulp for exp on its
normal range and 2 ulp for log.
"""

import numpy as np


def _ulp_error(got, exact):
    ref = exact.astype(np.float32)
    spacing = np.abs(np.spacing(ref)).astype(np.float64)
    return np.abs(got.astype(np.float64) - exact) / spacing


def test_exp_within_one_ulp(oracle):
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.uniform(-87.0, 88.0, 200_000),
        rng.uniform(-6.0, 0.0, 200_000),  # the compositing range
        np.array([0.0, -0.5, 1.0, -1.0, 10.0, -10.0]),
    ]).astype(np.float32)
    got = oracle.exp(x)
    err = _ulp_error(got, np.exp(x.astype(np.float64)))
    assert err.max() <= 1.0, err.max()


def test_exp_special_values(oracle):
    x = np.array([np.nan, np.inf, -np.inf, 100.0, -200.0, -100.0], np.float32)
    y = oracle.exp(x)
    assert np.isnan(y[0]) and y[1] == np.inf and y[2] == 0.0 and y[3] == np.inf
    assert y[4] == 0.0
    assert 0.0 < y[5] < 1e-40  # subnormal range still produces a value


def test_log_within_two_ulp(oracle):
    rng = np.random.default_rng(1)
    x = np.concatenate([
        np.exp(rng.uniform(-80.0, 80.0, 200_000)),
        rng.uniform(0.5, 2.0, 200_000),
        rng.uniform(1.0, 255.0, 100_000),  # log(255 * opacity)
    ]).astype(np.float32)
    got = oracle.log(x)
    err = _ulp_error(got, np.log(x.astype(np.float64)))
    assert err.max() <= 2.0, err.max()


def test_log_special_values(oracle):
    x = np.array([0.0, -1.0, np.nan, np.inf, 1.0, 1e-40], np.float32)
    y = oracle.log(x)
    assert y[0] == -np.inf and np.isnan(y[1]) and np.isnan(y[2]) and y[3] == np.inf
    assert y[4] == 0.0
    assert abs(float(y[5]) - np.log(np.float64(np.float32(1e-40)))) < 1e-4
