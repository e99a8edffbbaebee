"""Splat relocation for MCMC-style training, on the GPU.

Same functions, arguments and behaviour as the reference's training helpers
(``training/utils.py:104-210``): ``relocate_splats`` replaces nearly
transparent splats (opacity < 0.005) with copies of visible ones sampled by
opacity, optionally densifies by appending copies, and zeroes the Adam moments
of every row it touched. The random draws are the reference's own
(``torch.multinomial`` in :func:`sample_counts`, same calls in the same order);
everything after them -- ``copy_splats`` with its ``normalize_copies``
(training/utils.py:94-101,120-145) and the optimizer-state reset -- is one
``gs_relocate`` pass instead of a host round trip (``counts.cpu()``), a dozen
gathers and scatters and a ``unique``.

The renormalised opacity and scale are computed in double precision and
rounded once; the reference chains float32 operations, so its values differ
from these by its own rounding (largest for many copies: the alternating
binomial series of normalize_copies cancels). Positions, rotations, colours,
normals and moments are copied or zeroed exactly.

Differences: ``relocate_splats`` raises ``TypeError`` for an unsupported
optimizer before touching the splats (the reference raises after editing
them), and there is no CPU path.
"""

from __future__ import annotations

import ctypes

import torch

from . import native
from .splats import GaussianSplat

PARAMETER_NAMES = ("mean", "rotation", "scale", "opacity", "color")
_ALL_NAMES = PARAMETER_NAMES + ("normals",)
_DEAD_OPACITY = 0.005  # training/utils.py:158


def sample_counts(weights: torch.Tensor, count: int) -> torch.Tensor:
    """How many copies each row gets: ``count`` draws with replacement,
    weighted by ``weights`` (training/utils.py:104-107)."""
    indices = torch.multinomial(weights, count, replacement=True)
    return torch.bincount(indices, minlength=len(weights))


def append_empty_splats(splats: GaussianSplat, count: int) -> GaussianSplat:
    """A new splat set of ``count`` more zero rows (training/utils.py:110-117)."""
    extended = GaussianSplat(0, sh_degree=splats.sh_degree).to(splats.mean)
    for name in _ALL_NAMES:
        value = getattr(splats, name)
        value = torch.cat((value.detach(), value.new_zeros(count, *value.shape[1:])))
        setattr(extended, name, torch.nn.Parameter(value))
    return extended


def _device_tensor(t: torch.Tensor, name: str, dtype: torch.dtype) -> torch.Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"relocation runs on CUDA devices only (there is no CPU path); "
                           f"{name} is on {t.device}")
    if t.dtype != dtype or not t.is_contiguous():
        raise RuntimeError(f"relocation needs {name} as a contiguous {dtype} tensor, got "
                           f"{t.dtype}{'' if t.is_contiguous() else ' (not contiguous)'}")
    return t


def _moments(optimizer, params) -> tuple[native.SplatArrays | None, ...]:
    """gs_splat_arrays of exp_avg and exp_avg_sq for the five parameters
    (NULL members where the optimizer holds no state yet)."""
    if optimizer is None:
        return None, None
    sets = []
    for key in ("exp_avg", "exp_avg_sq"):
        pointers = []
        for name, p in zip(PARAMETER_NAMES, params):
            value = optimizer.state.get(p, {}).get(key)
            if value is not None:
                _device_tensor(value, f"{name} {key}", torch.float32)
                if value.shape != p.shape:
                    raise RuntimeError(f"{name} {key} has shape {tuple(value.shape)}, "
                                       f"parameter {tuple(p.shape)}")
            pointers.append(None if value is None else value.data_ptr())
        sets.append(native.SplatArrays(*pointers))
    return tuple(sets)


def _relocate(splats: GaussianSplat, counts: torch.Tensor, output_indices: torch.Tensor | None,
              output_base: int, num_outputs: int, moments) -> torch.Tensor:
    """Launch gs_relocate on ``splats``; returns its workspace (for the
    status read)."""
    params = [_device_tensor(getattr(splats, name).data, name, torch.float32)
              for name in PARAMETER_NAMES]
    device = params[0].device
    counts = _device_tensor(counts.to(device=device, dtype=torch.int64).contiguous(),
                            "counts", torch.int64)
    if output_indices is not None:
        output_indices = _device_tensor(
            output_indices.to(device=device, dtype=torch.int64).contiguous(),
            "output_indices", torch.int64)
    normals = getattr(splats, "normals", None)
    if normals is not None:
        normals = _device_tensor(normals.data, "normals", torch.float32)
    lib = native.lib()
    size = int(lib.gs_relocate_workspace_size(len(counts)))
    workspace = torch.empty((size,), dtype=torch.uint8, device=device)
    arrays = native.SplatArrays(*(p.data_ptr() for p in params))
    exp_avg, exp_avg_sq = moments
    with torch.cuda.device(device):
        stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        native.check(lib.gs_relocate(
            len(counts), len(params[0]), params[4].shape[1], ctypes.c_void_p(counts.data_ptr()),
            num_outputs,
            ctypes.c_void_p(None if output_indices is None else output_indices.data_ptr()),
            output_base, ctypes.byref(arrays),
            ctypes.c_void_p(None if normals is None else normals.data_ptr()),
            None if exp_avg is None else ctypes.byref(exp_avg),
            None if exp_avg_sq is None else ctypes.byref(exp_avg_sq),
            ctypes.c_void_p(workspace.data_ptr()), size, stream), "gs_relocate")
    return workspace


def _check(workspace: torch.Tensor) -> None:
    with torch.cuda.device(workspace.device):
        stream = ctypes.c_void_p(torch.cuda.current_stream(workspace.device).cuda_stream)
        native.check(native.lib().gs_relocate_status(ctypes.c_void_p(workspace.data_ptr()),
                                                     stream),
                     "gs_relocate (counts must be >= 0 and add up to the number of output "
                     "rows, output rows inside the splat set)")


@torch.no_grad()
def copy_splats(splats: GaussianSplat, counts: torch.Tensor,
                output_indices: torch.Tensor) -> torch.Tensor:
    """In-place copy of parents (rows with counts > 0) to ``output_indices``
    with normalize_copies applied to parents and copies (training/utils.py:
    120-145). Returns the sorted unique parent and output rows, as the
    reference does."""
    if len(output_indices) != int(counts.sum()):
        raise RuntimeError(f"counts add up to {int(counts.sum())} copies for "
                           f"{len(output_indices)} output rows")
    _check(_relocate(splats, counts, output_indices, 0, len(output_indices), (None, None)))
    parents = counts.nonzero().squeeze(-1).to(output_indices.device)
    return torch.cat((parents, output_indices)).unique()


@torch.no_grad()
def _move_optimizer_state(optimizer, replacement: dict, extra_rows: int) -> None:
    """Hands each replaced parameter's optimizer state to its replacement.

    ``replacement`` maps id(old parameter) to the new, ``extra_rows`` longer
    parameter. The state dict is re-keyed to the new tensor with both Adam
    moments padded by zero rows, and every parameter group is rebuilt to refer
    to the new tensors (training/utils.py:195-209 does the same bookkeeping)."""
    for old_id, new in replacement.items():
        old = next((p for p in optimizer.state if id(p) == old_id), None)
        if old is None:
            continue
        state = optimizer.state.pop(old)

        def padded(value):
            return torch.cat((value, value.new_zeros((extra_rows, *value.shape[1:]))))

        optimizer.state[new] = {key: padded(value) if key in ("exp_avg", "exp_avg_sq") else value
                                for key, value in state.items()}
    for group in optimizer.param_groups:
        group["params"] = [replacement.get(id(p), p) for p in group["params"]]


def relocate_splats(splats: GaussianSplat, optimizer: torch.optim.Optimizer | None = None,
                    densification_factor: float = 1.0) -> None:
    """Replace dead splats with sampled copies of live ones, densify to
    ``densification_factor`` times the current count, and reset the Adam
    moments of every touched row (training/utils.py:147-210). With an
    optimizer, densified parameters replace the old ones in its groups and
    state, as in the reference."""
    if optimizer is not None and not isinstance(optimizer, (torch.optim.Adam,
                                                            torch.optim.AdamW)):
        raise TypeError("optimizer must be Adam, AdamW, or None")
    n = len(splats.mean)
    params = [getattr(splats, name) for name in PARAMETER_NAMES]
    extra_states = [] if optimizer is None else [
        state for p, state in optimizer.state.items() if not any(p is q for q in params)]
    workspaces, reset = [], []

    # Replace nearly transparent splats with copies of visible ones
    opacity = splats.opacity.sigmoid().squeeze(-1)
    dead_mask = opacity < _DEAD_OPACITY
    dead_indices = dead_mask.nonzero().squeeze(-1)
    if 0 < len(dead_indices) < len(opacity):
        counts = sample_counts(opacity.masked_fill(dead_mask, 0), len(dead_indices))
        workspaces.append(_relocate(splats, counts, dead_indices, 0, len(dead_indices),
                                    _moments(optimizer, params)))
        if extra_states:
            reset += [counts.nonzero().squeeze(-1), dead_indices]

    # Densify if needed
    target = int(densification_factor * n)
    diff = max(0, target - n)
    if diff:
        opacity = splats.opacity.sigmoid().squeeze(-1)
        extended = append_empty_splats(splats, diff)
        counts = sample_counts(opacity, diff)
        if optimizer is not None:
            # Grow the moments first (zero rows for the new splats), so the
            # kernel resets the parents' rows in the grown state.
            _move_optimizer_state(optimizer, {id(getattr(splats, name)): getattr(extended, name)
                                              for name in _ALL_NAMES}, diff)
        new_params = [getattr(extended, name) for name in PARAMETER_NAMES]
        workspaces.append(_relocate(extended, counts, None, n, diff,
                                    _moments(optimizer, new_params)))
        if extra_states:
            reset.append(counts.nonzero().squeeze(-1))
        for name in _ALL_NAMES:
            setattr(splats, name, getattr(extended, name))

    # Optimizer state of parameters other than the five (e.g. normals, if
    # trained): zeroed at the touched rows, as the reference does for every
    # state it holds.
    if extra_states and reset:
        indices = torch.cat(reset).unique()
        for state in extra_states:
            for key in ("exp_avg", "exp_avg_sq"):
                if key in state:
                    state[key][indices] = 0
    for workspace in workspaces:
        _check(workspace)
