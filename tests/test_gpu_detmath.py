"""The kernels' exp / log agree bit for bit with the oracle's copy.

Integer outputs (tile bounds, counts, contributor counts) are only bit-exact
against the oracle because both sides evaluate the same exp/log algorithm
with the same IEEE float32 operations; this checks the CUDA build of that
algorithm (gs_det_exp / gs_det_log through the C ABI) over a dense sweep.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _device_apply(name, x):
    from gaussian_splats_b200 import native

    lib = native.lib()
    d_x = torch.from_numpy(x).cuda()
    d_y = torch.empty_like(d_x)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    native.check(getattr(lib, name)(x.size, ctypes.c_void_p(d_x.data_ptr()),
                                    ctypes.c_void_p(d_y.data_ptr()), stream), name)
    return d_y.cpu().numpy()


def _sweep():
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2**32, 4_000_000, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    extra = np.concatenate([
        np.linspace(-110, 90, 1_000_001, dtype=np.float32),
        np.linspace(-6, 0, 1_000_001, dtype=np.float32),
        np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45], np.float32),
    ])
    return np.concatenate([x, extra]).astype(np.float32)


def _same_bits(a, b):
    a_nan, b_nan = np.isnan(a), np.isnan(b)
    assert np.array_equal(a_nan, b_nan)
    return np.array_equal(a[~a_nan].view(np.uint32), b[~b_nan].view(np.uint32))


def test_exp_bitwise(oracle):
    x = _sweep()
    assert _same_bits(_device_apply("gs_det_exp", x), oracle.exp(x))


def test_log_bitwise(oracle):
    x = np.abs(_sweep())
    assert _same_bits(_device_apply("gs_det_log", x), oracle.log(x))
