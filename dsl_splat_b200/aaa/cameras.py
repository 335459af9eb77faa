"""OpenCV pinhole cameras lowered to AAA's kernel parameters
(aaa/cameras.py:44-121).

The lowering is Torch arithmetic on the caller's tensors, so pose gradients
flow back to viewmats through it: the transposed view matrix, the full
projection (P V)^T with AAA's frontend projection (nominal near/far mapped to
depth 0/1) and the camera centres from the inverse views.  The intrinsics are
read once on the host, as the reference does.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import Tensor

from ..cameras import read_intrinsics
from .stages import AaaView


def _camera_matmul(left: Tensor, right: Tensor) -> Tensor:
    """float32 camera products even under autocast (runtime/precision.py:7-12)."""
    if torch.is_autocast_enabled():
        with torch.autocast(device_type="cuda", enabled=False):
            return left @ right
    return left @ right


@dataclass(slots=True)
class CameraBatch:
    transposed_views: Tensor   # (B,C,4,4)
    projection: Tensor         # (B,C,4,4) (P V)^T
    centers: Tensor            # (B,C,3)
    intrinsics: list           # per batch, per camera (fx, fy, cx, cy)
    width: int
    height: int

    def view(self, batch: int, camera: int) -> AaaView:
        """aaa/cameras.py:52-75 config: tanfov = size / (2 f), principal point (cx, cy)."""
        fx, fy, cx, cy = self.intrinsics[batch][camera]
        return AaaView(self.width, self.height, self.width / (2 * fx), self.height / (2 * fy),
                       (cx, cy), self.transposed_views[batch, camera],
                       self.projection[batch, camera], self.centers[batch, camera])


def prepare_cameras(viewmats: Tensor, Ks: Tensor, width: int, height: int, near_plane: float,
                    far_plane: float) -> CameraBatch:
    """aaa/cameras.py:78-121 for (B,C,4,4) viewmats and (B,C,3,3) Ks."""
    batch_count, cameras = viewmats.shape[0], viewmats.shape[1]
    intrinsics = read_intrinsics(Ks)
    inverse_views = torch.linalg.inv(viewmats)
    p = torch.zeros(batch_count, cameras, 4, 4, dtype=torch.float32)
    p[..., 0, 0] = 2 * intrinsics[..., 0, 0] / width
    p[..., 1, 1] = 2 * intrinsics[..., 1, 1] / height
    p[..., 0, 2] = 2 * intrinsics[..., 0, 2] / width - 1
    p[..., 1, 2] = 2 * intrinsics[..., 1, 2] / height - 1
    p[..., 2, 2] = 1 if math.isinf(far_plane) else far_plane / (far_plane - near_plane)
    p[..., 2, 3] = (-near_plane if math.isinf(far_plane)
                    else -far_plane * near_plane / (far_plane - near_plane))
    p[..., 3, 2] = 1
    full = _camera_matmul(p.to(viewmats.device), viewmats).transpose(-1, -2).contiguous()
    values = [[(k[0][0], k[1][1], k[0][2], k[1][2]) for k in batch]
              for batch in intrinsics.tolist()]
    return CameraBatch(viewmats.transpose(-1, -2).contiguous(), full,
                       inverse_views[..., :3, 3].contiguous(), values, width, height)


__all__ = ["CameraBatch", "prepare_cameras"]
