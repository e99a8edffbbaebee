"""Rendering and training steps replayed from CUDA graphs.

A step of the reference's training loop (training/train.py:125-151: render,
loss, backward) launches about twenty kernels and runs a few hundred
microseconds of Python per view; for small scenes the host, not the GPU, sets
the pace. :class:`CapturedStep` captures such a step once as a CUDA graph and
replays it: one launch per step, no Python in the loop.

The rasterizer's forward normally waits once per render for the number of
tile intersections, which sizes its sort buffer and the ``gaussian_ids``
output. Under capture it cannot wait, so it sorts into a buffer sized from
the eager warm-up renders (plus ``headroom``), its ``gaussian_ids`` output
keeps that capacity (entries past the tile ranges are unused), and a copy
inside the graph leaves each render's true total and error word in pinned
host memory. :meth:`CapturedStep.check` reads them after a replay; if a view
needed more room than it had, the results of that replay are invalid, so the
step is captured again with larger buffers and replayed before ``check``
returns.

Rules for the step function: it must work on static tensors (the same splat
parameters, camera and target objects every call; copy new values into them
in place between replays), render every view on the same devices and image
sizes each call, and keep host-side decisions out of the step (no ``.item()``
or other reads of device values). Camera poses are read from device tensors
the graph captured: keep the camera's quaternion and translation on the GPU,
or re-render a changed host camera eagerly before capturing. Set the
parameters' ``.grad`` to None at the start of the step (``train_step`` does):
the captured backward then writes fresh gradients into tensors the graph owns
on every replay instead of adding to old ones; nothing may reset them between
replays. The optimizer step (whose scalars change with the step count) and
relocation stay outside the graph, and so do collectives: a step that
exchanges gradients across ranks (``view_parallel``) is refused after its
warm-up and stays launched from Python.
"""

from __future__ import annotations

from collections.abc import Callable

import torch

from . import rasterize as _rasterize
from . import view_parallel

_HEADROOM_SLACK = 4096  # intersections added to every capacity


class _Capture:
    """Bookkeeping of one capture: intersection capacities per render shape,
    pinned result words handed to each render, and what each render got."""

    def __init__(self, capacities: dict, words: list[torch.Tensor], headroom: float):
        self.capacities = capacities
        self.words = words
        self.headroom = headroom
        self.renders: list[tuple[tuple, int, torch.Tensor]] = []
        self.kept: list[torch.Tensor] = []

    def keep(self, host_buffer: torch.Tensor) -> None:
        """Hold a pinned host buffer a captured copy reads on every replay."""
        self.kept.append(host_buffer)

    def capacity(self, key, last: int) -> int:
        if key not in self.capacities:
            self.capacities[key] = last + int(last * self.headroom) + _HEADROOM_SLACK
        return self.capacities[key]

    def take_words(self) -> torch.Tensor:
        if len(self.renders) >= len(self.words):
            raise RuntimeError(f"more than {len(self.words)} renders in one captured step; "
                               "raise max_renders")
        words = self.words[len(self.renders)]
        words.zero_()
        return words

    def record(self, key, capacity: int, words: torch.Tensor) -> None:
        self.renders.append((key, capacity, words))


class CapturedStep:
    """``fn`` (a step on static tensors returning a tensor, e.g. the loss)
    captured as a CUDA graph; calling the object replays it.

    ``fn`` runs eagerly ``warmup`` times on a side stream first (as CUDA-graph
    capture of autograd requires), which also sizes every render's
    intersection buffer; ``headroom`` is the fraction added on top. Each call
    replays the graph and returns ``fn``'s output tensor (the same tensor,
    overwritten by every replay). Call :meth:`check` after a replay, before
    using its results, whenever the views can change between replays.
    """

    def __init__(self, fn: Callable[[], torch.Tensor], warmup: int = 2, headroom: float = 0.25,
                 max_renders: int = 64):
        if warmup < 1:
            raise ValueError("warmup must be at least 1 (it sizes the intersection buffers)")
        self.fn = fn
        self.headroom = headroom
        self.capacities: dict = {}
        self.words = [torch.zeros(2, dtype=torch.int64, pin_memory=True)
                      for _ in range(max_renders)]
        self.graph: torch.cuda.CUDAGraph | None = None
        self.output: torch.Tensor | None = None
        self.renders: list = []
        self.captures = 0
        self._capture(warmup)

    def _capture(self, warmup: int) -> None:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        collectives = view_parallel.COLLECTIVE_CALLS
        seen: dict = {}
        previous_seen, _rasterize._SEEN_TOTALS = _rasterize._SEEN_TOTALS, seen
        try:
            with torch.cuda.stream(side):
                for _ in range(warmup):
                    self.fn()
        finally:
            _rasterize._SEEN_TOTALS = previous_seen
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        if view_parallel.COLLECTIVE_CALLS != collectives:
            # Decided from the eager warm-up, the same on every rank: capturing
            # the step's NCCL collectives into a graph hung on two GPUs here.
            raise RuntimeError("the step exchanges gradients across ranks; launch it from "
                               "Python (collectives are not captured into CUDA graphs)")
        # every render of a shape gets room for the largest one seen
        for key, total in seen.items():
            self._grow(key, total)
        self.graph = None  # release the previous graph's memory first
        graph = torch.cuda.CUDAGraph()
        capture = _Capture(self.capacities, self.words, self.headroom)
        previous, _rasterize._CAPTURE = _rasterize._CAPTURE, capture
        try:
            with torch.cuda.graph(graph):
                output = self.fn()
        finally:
            _rasterize._CAPTURE = previous
        self.graph, self.output, self.renders = graph, output, capture.renders
        self._kept = capture.kept  # host buffers the graph's copies read
        self.captures += 1

    def _grow(self, key, total: int) -> None:
        want = total + int(total * self.headroom) + _HEADROOM_SLACK
        self.capacities[key] = max(want, self.capacities.get(key, 0))

    def __call__(self) -> torch.Tensor:
        self.graph.replay()
        return self.output

    def check(self, retries: int = 3) -> bool:
        """Wait for the last replay and verify its renders. Returns True if
        every render fitted its buffer; otherwise re-captures with larger
        buffers, replays, and returns False once a replay fits (raises after
        ``retries`` attempts). Raises if a device-side wait gave up."""
        fitted = True
        for _ in range(retries + 1):
            torch.cuda.current_stream().synchronize()
            overflow = False
            for key, capacity, words in self.renders:
                total, error = int(words[0]), int(words[1]) & 0xFFFFFFFF
                if error:
                    raise RuntimeError(f"binning reported error word {error:#x} in a replay")
                if total >= 1 << 30:
                    raise RuntimeError(f"{total} intersections exceed the sort's capacity")
                if total > capacity:
                    overflow = True
                    self._grow(key, total)
            if not overflow:
                return fitted
            fitted = False
            self._capture(warmup=1)
            self.graph.replay()
        raise RuntimeError("captured step still overflows its intersection buffers")
