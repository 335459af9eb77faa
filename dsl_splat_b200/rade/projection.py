"""RaDe-GS projection stage (rade/projection.py:401-551 prepare/backward) on
the sm_100a kernels: one launch each way.

prepare writes centers, conics (with kernel_size dilation and opacity
compensation), radii, tile counts, radial sort distances, ray planes and
camera-space normals; rows with radii == 0 keep unspecified centers/conics/
planes/normals, as the reference leaves them unwritten.  backward is the VJP
of rade/projection.py:294-317 projection_loss with the reference's custom
adjoints; culled rows get explicit zeros.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from .. import stages
from .._native import check, lib, ptr
from ..camera_prep import ViewConfig as _SplatConfig


@dataclass(frozen=True, slots=True)
class ViewConfig(_SplatConfig):
    """rade/types.py:9-11: the shared view configuration plus kernel_size."""

    kernel_size: float = 0.0


@dataclass(slots=True)
class ProjectedGaussians(stages.ProjectedGaussians):
    """rade/types.py:14-17."""

    ray_planes: Tensor
    normals: Tensor


def prepare(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor, view: Tensor,
            projection: Tensor, intrinsics: Tensor, config: ViewConfig) -> ProjectedGaussians:
    """rade/projection.py:422-472 (quats already normalised)."""
    pin = stages.Args()
    n = len(means)
    dev = means.device
    state = ProjectedGaussians(means.new_empty((n, 2)), means.new_empty((n, 4)),
                               torch.empty(n, dtype=torch.int32, device=dev),
                               torch.empty(n, dtype=torch.int32, device=dev),
                               means.new_empty(n), means.new_empty((n, 3)),
                               means.new_empty((n, 3)))
    if n:
        check(lib.splat_rade_project_forward(
            n, pin(means), pin(quats), pin(scales), pin(opacities), pin(view), pin(projection),
            pin(intrinsics), config.width, config.height, float(config.near),
            stages._far(config.far), float(config.radius_clip), float(config.kernel_size),
            ptr(state.centers), ptr(state.conics), ptr(state.radii), ptr(state.tile_counts),
            ptr(state.depths), ptr(state.ray_planes), ptr(state.normals),
            stages._stream(means)), "rade_project_forward")
    return state


def backward(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor, view: Tensor,
             projection: Tensor, intrinsics: Tensor, config: ViewConfig,
             state: ProjectedGaussians, grad_centers: Tensor | None,
             grad_conics: Tensor | None, grad_planes: Tensor | None,
             grad_normals: Tensor | None, needs: tuple[bool, ...]) -> list[Tensor | None]:
    """rade/projection.py:475-551: [means, quats, scales, opacities, view,
    projection] gradients (None where needs is False)."""
    if not any(needs):
        return [None] * 6
    pin = stages.Args()
    tensors = [means, quats, scales, opacities]
    grads = [torch.empty_like(t) if need else None for t, need in zip(tensors, needs[:4])]
    n = len(means)
    cam = means.new_zeros(32) if any(needs[4:]) else None
    if n:
        check(lib.splat_rade_project_backward(
            n, pin(means), pin(quats), pin(scales), pin(opacities), pin(view), pin(projection),
            pin(intrinsics), config.width, config.height, float(config.kernel_size),
            ptr(state.radii), pin(grad_centers), pin(grad_conics), pin(grad_planes),
            pin(grad_normals), *[ptr(g) for g in grads],
            ptr(None if cam is None else cam[:16]), ptr(None if cam is None else cam[16:]),
            stages._stream(means)), "rade_project_backward")
    out: list[Tensor | None] = grads + [None, None]
    if needs[4]:
        out[4] = cam[:16].reshape(4, 4)
    if needs[5]:
        out[5] = cam[16:].reshape(4, 4)
    return out
