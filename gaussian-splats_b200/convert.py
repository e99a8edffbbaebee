"""Checkpoint <-> PLY conversion, the two commands of the reference's
``splats/convert.py`` (``pt-to-ply``, ``ply-to-pt``) as functions.

The reference wraps them in a typer CLI; a CLI is outside this package's
scope, so callers (or a one-line ``python -c``) use the functions directly.
Checkpoints are ``GaussianSplat.state_dict()`` files (``splats/splats.py``),
PLY files the layout of :mod:`gaussian_splats_b200.ply`.
"""

from __future__ import annotations

from pathlib import Path

from .ply import load_ply, save_ply
from .splats import GaussianSplat


def pt_to_ply(checkpoint: str | Path, output: str | Path | None = None) -> Path:
    """Write the splats of a checkpoint as PLY (convert.py ``pt-to-ply``);
    ``output`` defaults to the checkpoint path with a ``.ply`` suffix."""
    checkpoint = Path(checkpoint)
    output = Path(output) if output is not None else checkpoint.with_suffix(".ply")
    save_ply(GaussianSplat.from_checkpoint(checkpoint).state_dict(), output)
    return output


def ply_to_pt(ply: str | Path, output: str | Path | None = None) -> Path:
    """Write the splats of a PLY file as a checkpoint (convert.py
    ``ply-to-pt``); ``output`` defaults to the PLY path with a ``.pt`` suffix."""
    ply = Path(ply)
    output = Path(output) if output is not None else ply.with_suffix(".pt")
    GaussianSplat.from_tensors(**load_ply(ply)).save_checkpoint(output)
    return output
