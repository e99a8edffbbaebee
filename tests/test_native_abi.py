"""The C-ABI library loads and exports every entry point its header declares.

No GPU needed: only symbol lookup and the host-side workspace-size queries run.
"""

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "gs_b200.h")


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gs_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from gaussian_splats_b200 import native

    if not os.path.exists(native.LIBRARY_PATH):
        import __graft_entry__

        __graft_entry__.build()
    return native.lib()


def test_header_declares_the_bound_symbols():
    from gaussian_splats_b200 import native

    assert _declared_functions() == sorted(native.EXPORTED_SYMBOLS)


def test_every_declared_symbol_is_exported(lib):
    handle = ctypes.CDLL(lib._name)
    for name in _declared_functions():
        assert hasattr(handle, name), name


def test_version(lib):
    assert lib.gs_version() == 100


def test_workspace_sizes(lib):
    from gaussian_splats_b200 import native

    # Grow with the problem, stay 256-byte granular, and are pure host queries.
    small = lib.gs_bin_count_workspace_size(1000)
    large = lib.gs_bin_count_workspace_size(1_000_000)
    assert 0 < small < large and small % 256 == 0 and large % 256 == 0
    # Count phase holds 4 arrays of n 32-bit words plus per-tile status.
    assert large >= 16 * 1_000_000
    # Sort phase: a 1920x1088 view at 16x16 tiles (the row/column path holds
    # a segment array of the capacity), and a grid too wide for its tables
    # (the radix path: keys and values twice over).
    wide = native.make_params(500.0, 500.0, 4160.0, 8.0, 8320, 16, 4, 0.999, 0.2, 100.0,
                              "gaussian", 0.95)
    view = native.make_params(1000.0, 1000.0, 960.0, 540.0, 1920, 1088, 16, 0.999, 0.2, 100.0,
                              "gaussian", 0.95)
    s0 = lib.gs_bin_sort_workspace_size(1_000_000, 0, ctypes.byref(view))
    s1 = lib.gs_bin_sort_workspace_size(1_000_000, 5_000_000, ctypes.byref(view))
    assert s0 < s1 and s1 >= 4 * 5_000_000
    w1 = lib.gs_bin_sort_workspace_size(1_000_000, 5_000_000, ctypes.byref(wide))
    assert w1 >= 16 * 5_000_000
    assert lib.gs_bin_sort_workspace_size(1000, 1000, None) == 0  # invalid parameters
    assert lib.gs_bin_count_workspace_size(0) > 0


def test_argument_checks_without_gpu(lib):
    """Invalid arguments are rejected before anything touches a device."""
    from gaussian_splats_b200 import native

    p = native.make_params(10.0, 10.0, 8.0, 8.0, 16, 16, 3, 0.999, 0.2, 100.0, "gaussian", 0.95)
    null = ctypes.c_void_p(0)
    status = lib.gs_project_fwd(1, 1, *([null] * 7), ctypes.byref(p), *([null] * 7), null)
    assert status == -1  # tile size 3
    p = native.make_params(10.0, 10.0, 8.0, 8.0, 16, 16, 8, 0.999, 0.2, 100.0, "gaussian", 0.95)
    status = lib.gs_project_fwd(1, 36, *([null] * 7), ctypes.byref(p), *([null] * 7), null)
    assert status == -4  # SH degree 5
    total = ctypes.c_int64(0)
    status = lib.gs_bin_count(10, null, null, null, 0, ctypes.byref(total), null)
    assert status == -1  # workspace too small
