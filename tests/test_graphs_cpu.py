"""Host bookkeeping of captured steps (gaussian_splats_b200.graphs): buffer
capacities per render shape and the pinned result words handed to renders."""

import pytest
import torch

from gaussian_splats_b200 import graphs


def test_capacity_from_the_last_total_then_fixed():
    capture = graphs._Capture({}, [torch.zeros(2, dtype=torch.int64)] * 2, headroom=0.25)
    key = (1000, 300, 0)
    first = capture.capacity(key, 10_000)
    assert first == 10_000 + 2_500 + graphs._HEADROOM_SLACK
    assert capture.capacity(key, 99_999) == first  # one capacity per shape and capture


def test_words_run_out_with_a_clear_error():
    words = [torch.ones(2, dtype=torch.int64) for _ in range(2)]
    capture = graphs._Capture({}, words, headroom=0.25)
    for i in range(2):
        w = capture.take_words()
        assert torch.count_nonzero(w) == 0  # handed out zeroed
        capture.record(("k",), 10, w)
    with pytest.raises(RuntimeError, match="raise max_renders"):
        capture.take_words()
    assert [r[1] for r in capture.renders] == [10, 10]


def test_growth_keeps_the_largest_need():
    step = graphs.CapturedStep.__new__(graphs.CapturedStep)  # bookkeeping only, no capture
    step.headroom, step.capacities = 0.25, {}
    step._grow("a", 40_000)
    step._grow("a", 10_000)  # a smaller view of the same shape never shrinks it
    assert step.capacities["a"] == 40_000 + 10_000 + graphs._HEADROOM_SLACK


def test_kept_host_buffers():
    capture = graphs._Capture({}, [], headroom=0.0)
    buffer = torch.zeros(17, dtype=torch.int32)
    capture.keep(buffer)
    assert capture.kept == [buffer]
