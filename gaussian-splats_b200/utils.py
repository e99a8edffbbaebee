"""Host-side helpers shared by the camera and splat containers.

These mirror the conventions of ``splats/utils.py`` in the reference
(``quaternion_to_rotation_matrix`` at splats/utils.py:8-25, ``rgb_to_sh`` at
splats/utils.py:28-29): quaternions are ``(w, x, y, z)`` and the SH DC term is
stored as ``(rgb - 0.5) / C0``.
"""

from __future__ import annotations

import torch

SH_C0 = 0.28209479177387814


def quaternion_to_rotation_matrix(quaternion: torch.Tensor) -> torch.Tensor:
    """Rotation matrix of a unit ``(w, x, y, z)`` quaternion, shape ``[..., 3, 3]``.

    Same entry formulas and evaluation order as splats/utils.py:8-25, so a
    camera built here hands the operator the same float32 matrix bits.
    """
    w, x, y, z = quaternion.unbind(dim=-1)
    rows = (
        1 - 2 * (y.square() + z.square()),
        2 * (x * y - w * z),
        2 * (x * z + w * y),
        2 * (x * y + w * z),
        1 - 2 * (x.square() + z.square()),
        2 * (y * z - w * x),
        2 * (x * z - w * y),
        2 * (y * z + w * x),
        1 - 2 * (x.square() + y.square()),
    )
    return torch.stack(rows, dim=-1).reshape(*quaternion.shape[:-1], 3, 3)


def rgb_to_sh(rgb: torch.Tensor) -> torch.Tensor:
    """DC SH coefficient whose evaluated colour is ``rgb`` (splats/utils.py:28-29)."""
    return (rgb - 0.5) / SH_C0


def sh_to_rgb(sh: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`rgb_to_sh`."""
    return sh * SH_C0 + 0.5


def quaternion_from_rotation(rotation: torch.Tensor) -> torch.Tensor:
    """Unit ``(w, x, y, z)`` quaternion of a 3x3 rotation matrix.

    Shepperd's method: take the largest of the four squared components
    (trace-based ``w`` or one of the diagonal-based ``x, y, z``) to avoid
    dividing by a small number, then read the other three from the
    off-diagonal sums/differences.
    """
    r = rotation.double()
    m00, m01, m02 = r[0, 0], r[0, 1], r[0, 2]
    m10, m11, m12 = r[1, 0], r[1, 1], r[1, 2]
    m20, m21, m22 = r[2, 0], r[2, 1], r[2, 2]
    candidates = torch.stack(
        (
            1 + m00 + m11 + m22,
            1 + m00 - m11 - m22,
            1 - m00 + m11 - m22,
            1 - m00 - m11 + m22,
        )
    )
    pick = int(torch.argmax(candidates))
    s = torch.sqrt(candidates[pick].clamp_min(1e-30)) * 2  # = 4 * |component|
    if pick == 0:
        q = (s / 4, (m21 - m12) / s, (m02 - m20) / s, (m10 - m01) / s)
    elif pick == 1:
        q = ((m21 - m12) / s, s / 4, (m01 + m10) / s, (m02 + m20) / s)
    elif pick == 2:
        q = ((m02 - m20) / s, (m01 + m10) / s, s / 4, (m12 + m21) / s)
    else:
        q = ((m10 - m01) / s, (m02 + m20) / s, (m12 + m21) / s, s / 4)
    q = torch.stack(q)
    q = q / q.norm()
    return q.to(rotation.dtype)
