"""Seeded synthetic scenes with the shapes and distributions of the benchmark configs.

There is no dataset here: every config is drawn from a CPU
``torch.Generator`` in a fixed order (means, log-scales, quaternions, opacity
logits, SH DC, SH rest, then cameras and targets), so any machine rebuilds the
same float32 inputs from the seed.

``config1`` .. ``config5`` follow the five benchmark configurations in order:
1. 16,384 Gaussians, SH0, 256x256, one view (the CPU-sized case);
2. 1M Gaussians, SH3, 1920x1080 (rendered 1920x1088), fwd+bwd, L1 loss;
3. 3M Gaussians (config-2 distributions), 8 cameras, 1600x1064 (1072);
4. 6M Gaussians, 3840x2160, 64-camera orbit, forward only;
5. 500k Gaussians in a dense blob, SH1, 1920x1080 (1088), fwd+bwd.
Heights that are not tile multiples are padded with the principal point kept
at the unpadded centre; crop results with ``[:height, :width]``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from .camera import PinholeCamera
from .utils import quaternion_from_rotation, rgb_to_sh


@dataclass
class RenderSettings:
    tile_size: int = 16
    opacity_threshold: float = 0.999
    near: float = 0.2
    far: float = 100.0
    rendering_mode: str = "gaussian"
    confidence: float = 0.95


@dataclass
class Scene:
    """Gaussian tensors (CPU, float32), cameras and per-camera targets."""

    mean: torch.Tensor
    rotation: torch.Tensor
    scale: torch.Tensor
    opacity: torch.Tensor
    color: torch.Tensor
    cameras: list[PinholeCamera]
    crop: tuple[int, int]  # unpadded (width, height)
    settings: RenderSettings = field(default_factory=RenderSettings)
    targets: list[torch.Tensor] | None = None  # [height, width, 3] per camera
    backward: bool = True

    @property
    def num_points(self) -> int:
        return self.mean.shape[0]

    def tensors(self) -> tuple[torch.Tensor, ...]:
        return self.mean, self.rotation, self.scale, self.opacity, self.color


def look_at_camera(
    position,
    target=(0.0, 0.0, 0.0),
    *,
    fovy_degrees: float,
    width: int,
    height: int,
    tile_size: int = 16,
) -> PinholeCamera:
    """Pinhole camera at ``position`` looking at ``target``.

    Rows of the world-to-camera matrix are (right, up, -forward); ``up`` is
    world +Z unless the view axis is nearly vertical, then world +Y. Focal
    length is ``(height / 2) / tan(fovy / 2)`` for both axes; the image is
    padded to a tile multiple with the principal point at the unpadded centre.
    """
    position = torch.as_tensor(position, dtype=torch.float64)
    target = torch.as_tensor(target, dtype=torch.float64)
    forward = target - position
    forward = forward / forward.norm()
    world_up = torch.tensor([0.0, 0.0, 1.0], dtype=torch.float64)
    if abs(float(forward @ world_up)) > 0.99:
        world_up = torch.tensor([0.0, 1.0, 0.0], dtype=torch.float64)
    right = torch.linalg.cross(forward, world_up)
    right = right / right.norm()
    up = torch.linalg.cross(right, forward)
    rotation = torch.stack((right, up, -forward))
    quaternion = quaternion_from_rotation(rotation).float()
    translation = (-(rotation @ position)).float()
    focal = (height / 2) / math.tan(math.radians(fovy_degrees) / 2)
    camera = PinholeCamera(
        rotation=quaternion,
        translation=translation,
        image_size=(width, height),
        focal_length=(focal, focal),
        principal_point=(width / 2, height / 2),
    )
    return camera.padded_to_tiles(tile_size)


def random_gaussians(
    generator: torch.Generator,
    num_points: int,
    *,
    means: tuple[str, float, float],
    log_scale: tuple[float, float],
    opacity_logit: tuple[float, float],
    sh_degree: int,
    sh_rest_std: float = 0.05,
) -> tuple[torch.Tensor, ...]:
    """Draw Gaussian tensors in the canonical order.

    ``means`` is ``("normal", mu, sigma)`` or ``("uniform", low, high)``.
    """
    kind, a, b = means
    if kind == "normal":
        mean = torch.randn(num_points, 3, generator=generator) * b + a
    else:
        mean = torch.rand(num_points, 3, generator=generator) * (b - a) + a
    scale = torch.randn(num_points, 3, generator=generator) * log_scale[1] + log_scale[0]
    rotation = torch.randn(num_points, 4, generator=generator)
    rotation = rotation / rotation.norm(dim=-1, keepdim=True)
    opacity = torch.randn(num_points, 1, generator=generator) * opacity_logit[1] + opacity_logit[0]
    k = (sh_degree + 1) ** 2
    color = torch.zeros(num_points, k, 3)
    color[:, 0, :] = rgb_to_sh(torch.rand(num_points, 3, generator=generator))
    if k > 1:
        color[:, 1:, :] = torch.randn(num_points, k - 1, 3, generator=generator) * sh_rest_std
    return mean, rotation, scale, opacity, color


def random_direction(generator: torch.Generator) -> torch.Tensor:
    v = torch.randn(3, generator=generator, dtype=torch.float64)
    return v / v.norm()


def _targets(generator, cameras, crop):
    width, height = crop
    return [torch.rand(height, width, 3, generator=generator) for _ in cameras]


def config1(num_points: int = 16_384, seed: int = 0, image: int = 256) -> Scene:
    g = torch.Generator().manual_seed(seed)
    tensors = random_gaussians(
        g,
        num_points,
        means=("uniform", -1.0, 1.0),
        log_scale=(-4.0, 0.5),
        opacity_logit=(0.0, 1.0),
        sh_degree=0,
    )
    camera = look_at_camera((0.0, 0.0, 4.0), fovy_degrees=60.0, width=image, height=image)
    settings = RenderSettings(near=0.01)
    return Scene(*tensors, cameras=[camera], crop=(image, image), settings=settings, backward=False)


def config2(
    num_points: int = 1_000_000, seed: int = 1, width: int = 1920, height: int = 1080,
    log_scale: tuple[float, float] = (-5.0, 0.7),
) -> Scene:
    g = torch.Generator().manual_seed(seed)
    tensors = random_gaussians(
        g,
        num_points,
        means=("normal", 0.0, 1.0),
        log_scale=log_scale,
        opacity_logit=(0.0, 1.5),
        sh_degree=3,
    )
    camera = look_at_camera(5.0 * random_direction(g), fovy_degrees=50.0, width=width, height=height)
    return Scene(*tensors, cameras=[camera], crop=(width, height),
                 targets=_targets(g, [camera], (width, height)))


def config3(
    num_points: int = 3_000_000, seed: int = 2, views: int = 8, width: int = 1600,
    height: int = 1064,
) -> Scene:
    g = torch.Generator().manual_seed(seed)
    tensors = random_gaussians(
        g,
        num_points,
        means=("normal", 0.0, 1.0),
        log_scale=(-5.0, 0.7),
        opacity_logit=(0.0, 1.5),
        sh_degree=3,
    )
    cameras = []
    for _ in range(views):
        radius = 4.0 + 2.0 * float(torch.rand(1, generator=g))
        cameras.append(look_at_camera(radius * random_direction(g), fovy_degrees=50.0,
                                      width=width, height=height))
    return Scene(*tensors, cameras=cameras, crop=(width, height),
                 targets=_targets(g, cameras, (width, height)))


def config4(
    num_points: int = 6_000_000, seed: int = 3, views: int = 64, width: int = 3840,
    height: int = 2160,
) -> Scene:
    g = torch.Generator().manual_seed(seed)
    tensors = random_gaussians(
        g,
        num_points,
        means=("uniform", -3.0, 3.0),
        log_scale=(-5.5, 0.5),
        opacity_logit=(0.0, 1.5),
        sh_degree=3,
    )
    cameras = []
    for i in range(views):
        angle = 2.0 * math.pi * i / views
        cameras.append(
            look_at_camera((6.0 * math.cos(angle), 6.0 * math.sin(angle), 0.0),
                           fovy_degrees=50.0, width=width, height=height)
        )
    return Scene(*tensors, cameras=cameras, crop=(width, height), backward=False)


def config5(
    num_points: int = 500_000, seed: int = 4, width: int = 1920, height: int = 1080,
) -> Scene:
    g = torch.Generator().manual_seed(seed)
    tensors = random_gaussians(
        g,
        num_points,
        means=("normal", 0.0, 0.2),
        log_scale=(-3.0, 0.5),
        opacity_logit=(-1.0, 1.0),
        sh_degree=1,
    )
    camera = look_at_camera((0.0, 0.0, 2.5), fovy_degrees=70.0, width=width, height=height)
    return Scene(*tensors, cameras=[camera], crop=(width, height),
                 targets=_targets(g, [camera], (width, height)))


CONFIGS = {"config1": config1, "config2": config2, "config3": config3, "config4": config4,
           "config5": config5}
