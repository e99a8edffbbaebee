"""Gaussian parameter container with the reference's tensor conventions.

Mirrors splats/splats.py:26-84. For ``N`` splats of SH degree ``d`` and
``K = (d + 1) ** 2``:

====================  ===========  =========================================
``mean``              N x 3        world-space centres
``rotation``          N x 4        ``(w, x, y, z)`` quaternions (any norm)
``scale``             N x 3        log standard deviations
``opacity``           N x 1        logits; alpha = sigmoid(opacity)
``color``             N x K x 3    real SH coefficients; evaluation adds 0.5
``normals``           N x 3        world-space normals (no gradient path)
====================  ===========  =========================================

Checkpoints are plain ``state_dict`` files with the same keys, so a file
written by either project loads in the other.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import torch
import torch.nn.functional as F
from torch import nn

from .utils import rgb_to_sh


@dataclass(frozen=True)
class ProjectedGaussianSplat:
    """Screen-space Gaussians (splats/splats.py:13-23)."""

    mean: torch.Tensor  # N x 3 (pixel x, pixel y, depth)
    covariance: torch.Tensor  # N x 2 x 2
    color: torch.Tensor  # N x 3
    opacity: torch.Tensor  # N x 1
    normals: torch.Tensor | None = None

    @property
    def inverse_covariance(self) -> torch.Tensor:
        return torch.linalg.inv(self.covariance)


class GaussianSplat(nn.Module):
    """Trainable Gaussian parameters (splats/splats.py:26-84)."""

    def __init__(self, num_points: int, sh_degree: int = 3):
        super().__init__()
        self.sh_degree = sh_degree
        self.mean = nn.Parameter(torch.randn(num_points, 3))
        self.rotation = nn.Parameter(F.normalize(torch.randn(num_points, 4)))
        self.scale = nn.Parameter(torch.randn(num_points, 3))
        self.opacity = nn.Parameter(torch.randn(num_points, 1))
        color = torch.zeros(num_points, (sh_degree + 1) ** 2, 3)
        color[:, 0, :] = rgb_to_sh(torch.rand(num_points, 3))
        self.color = nn.Parameter(color)
        self.normals = nn.Parameter(torch.zeros_like(self.mean))

    def save_checkpoint(self, path: str | Path) -> None:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        torch.save(self.state_dict(), path)

    @classmethod
    def from_checkpoint(cls, checkpoint: str | Path) -> "GaussianSplat":
        state = torch.load(checkpoint, map_location="cpu", weights_only=True)
        splats = cls(len(state["mean"]), int(state["color"].shape[1] ** 0.5) - 1)
        splats.load_state_dict(state)
        return splats

    @classmethod
    def from_tensors(
        cls,
        mean: torch.Tensor,
        rotation: torch.Tensor,
        scale: torch.Tensor,
        opacity: torch.Tensor,
        color: torch.Tensor,
        normals: torch.Tensor | None = None,
    ) -> "GaussianSplat":
        """Wrap existing tensors without the random initialisation cost."""
        splats = cls.__new__(cls)
        nn.Module.__init__(splats)
        splats.sh_degree = int(color.shape[1] ** 0.5) - 1
        with torch.no_grad():
            splats.mean = nn.Parameter(mean)
            splats.rotation = nn.Parameter(rotation)
            splats.scale = nn.Parameter(scale)
            splats.opacity = nn.Parameter(opacity)
            splats.color = nn.Parameter(color)
            splats.normals = nn.Parameter(
                normals if normals is not None else torch.zeros_like(mean)
            )
        return splats

    @property
    def num_points(self) -> int:
        return len(self.mean)
