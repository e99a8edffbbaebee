"""Camera types with the reference's conventions (splats/camera.py:14-144).

World-to-camera rotation (a ``(w, x, y, z)`` quaternion) and translation:
``p_camera = R @ p_world + t``. The camera looks down -Z with +Y up; pixel
coordinates grow right and down; focal lengths and the principal point are in
pixels.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field, replace

import torch
import torch.nn.functional as F

from .utils import quaternion_to_rotation_matrix


@dataclass(kw_only=True)
class Camera:
    """Base camera: pose and image size (splats/camera.py:14-52)."""

    rotation: torch.Tensor = field(default_factory=lambda: torch.tensor([1.0, 0.0, 0.0, 0.0]))
    translation: torch.Tensor = field(default_factory=lambda: torch.zeros(3))
    image_size: tuple[int, int] = (640, 480)

    # (quaternion tensor, its version, matrix, the matrix's version) of the
    # last rotation_matrix computed without autograd
    _matrix_cache: tuple | None = field(default=None, init=False, repr=False, compare=False)

    @property
    def rotation_matrix(self) -> torch.Tensor:
        """World-to-camera 3x3 matrix of the normalised quaternion.

        Remembered while the quaternion tensor is the same object with the same
        version counter (so in-place edits and reassignment recompute it): a
        render then pays no per-call torch ops for an unchanged camera.
        Quaternions that require grad are never cached, nor device quaternions
        during CUDA-graph capture (the graph must recompute the matrix from
        the quaternion on every replay)."""
        q = self.rotation
        if q.requires_grad or (q.is_cuda and torch.cuda.is_current_stream_capturing()):
            return quaternion_to_rotation_matrix(F.normalize(q, dim=-1))
        cache = self._matrix_cache
        if cache is not None and cache[0] is q and cache[1] == q._version and \
                cache[3] == cache[2]._version:
            return cache[2]
        matrix = quaternion_to_rotation_matrix(F.normalize(q, dim=-1))
        self._matrix_cache = (q, q._version, matrix, matrix._version)
        return matrix

    @property
    def position(self) -> torch.Tensor:
        """Camera centre in world space, ``-R^T t``."""
        return -(self.rotation_matrix.T @ self.translation)

    def to(self, device):
        self.rotation = self.rotation.to(device)
        self.translation = self.translation.to(device)
        return self

    @property
    def device(self) -> torch.device:
        return self.translation.device

    @property
    def dtype(self) -> torch.dtype:
        return self.translation.dtype


@dataclass(kw_only=True)
class PinholeCamera(Camera):
    """Pinhole camera (splats/camera.py:55-144)."""

    focal_length: tuple[float, float] = (500.0, 500.0)
    principal_point: tuple[float, float] = (320.0, 240.0)

    @property
    def intrinsics(self) -> torch.Tensor:
        fx, fy = self.focal_length
        cx, cy = self.principal_point
        return torch.tensor(
            [[fx, 0, -cx], [0, -fy, -cy], [0, 0, -1]], dtype=self.dtype, device=self.device
        )

    @torch.no_grad()
    def fit_to_points(self, points: torch.Tensor) -> "PinholeCamera":
        """Move the camera back along its view axis until ``points`` fit in view.

        Same framing rule as splats/camera.py:126-144: bounding-box centre, a
        radius of half the box diagonal, and a distance of
        ``1.1 * radius / sin(atan(tan_half_fov))`` with the narrower FOV.
        """
        self.to(points.device)
        if len(points) > 10_000:
            points = points[torch.randint(len(points), (10_000,), device=points.device)]
        lower, upper = torch.aminmax(points, dim=0)
        center = 0.5 * (lower + upper)
        radius = 0.5 * (upper - lower).norm().clamp_min(1e-3)
        fx, fy = self.focal_length
        width, height = self.image_size
        tan_half_fov = min(width / (2 * fx), height / (2 * fy))
        distance = 1.1 * radius / math.sin(math.atan(tan_half_fov))
        rotation = self.rotation_matrix
        position = center + distance * rotation[2]
        self.translation = -(rotation @ position)
        return self

    def padded_to_tiles(self, tile_size: int) -> "PinholeCamera":
        """Copy whose image size is rounded up to a multiple of ``tile_size``.

        The principal point stays at the centre of the unpadded image, which is
        how the reference renders sizes that are not tile multiples
        (visualize/gaussian/backend.py:25-27); crop the result back with
        ``image[:height, :width]``.
        """
        width, height = self.image_size
        padded = (
            (width + tile_size - 1) // tile_size * tile_size,
            (height + tile_size - 1) // tile_size * tile_size,
        )
        return replace(self, image_size=padded, principal_point=(width / 2, height / 2))
