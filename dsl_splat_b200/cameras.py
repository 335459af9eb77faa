"""OpenCV pinhole cameras and option validation (dsl_splat/cameras.py:1-62).

Same public names, error types and messages as the reference, so callers'
exception handling carries over unchanged.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from numbers import Integral

import torch
from torch import Tensor


def _positive_int(value) -> bool:
    return not isinstance(value, bool) and isinstance(value, Integral) and value > 0


def read_intrinsics(Ks: Tensor) -> Tensor:
    """Validate a small (...,3,3) intrinsic array on the host (cameras.py:11-27)."""
    k = Ks.cpu()
    if (not bool(torch.isfinite(k).all()) or bool((k[..., 0, 0] <= 0).any())
            or bool((k[..., 1, 1] <= 0).any())):
        raise ValueError("Ks must be finite with positive fx/fy")
    bottom = torch.tensor([0.0, 0.0, 1.0], dtype=torch.float32).expand(Ks.shape[:-2] + (3,))
    if (not torch.equal(k[..., 2, :], bottom) or bool((k[..., 0, 1] != 0).any())
            or bool((k[..., 1, 0] != 0).any())):
        raise NotImplementedError("Ks must be a zero-skew pinhole intrinsic matrix")
    return k


def validate_camera_options(width, height, near_plane, far_plane, radius_clip) -> None:
    """cameras.py:30-44: image size, clip planes and radius clip."""
    if not (_positive_int(width) and _positive_int(height)):
        raise ValueError("width and height must be positive integers")
    if (not math.isfinite(near_plane) or near_plane <= 0 or math.isnan(far_plane)
            or far_plane <= near_plane):
        raise ValueError("require 0 < near_plane < far_plane")
    if not math.isfinite(radius_clip) or radius_clip < 0:
        raise ValueError("radius_clip must be finite and nonnegative")


@dataclass(frozen=True, slots=True)
class PinholeCamera:
    """World-to-camera pose (OpenCV axes: right, down, forward) and zero-skew K."""

    viewmat: Tensor
    K: Tensor
    width: int
    height: int
    near_plane: float = 0.01
    far_plane: float = 1e10
