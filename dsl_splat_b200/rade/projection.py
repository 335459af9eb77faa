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


@dataclass(slots=True)
class FusedProjection:
    """The projection with the SH colours and the dense training metadata
    of the same launch (colors / active / metadata None when not asked)."""

    state: ProjectedGaussians
    colors: Tensor | None    # (n,3)
    active: Tensor | None    # (n,3) uint8 clamp mask
    means2d: Tensor | None   # (n,2), zero on culled rows
    opacities: Tensor | None
    conics3: Tensor | None   # (n,3)


def prepare_fused(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor, view: Tensor,
                  projection: Tensor, intrinsics: Tensor, config: ViewConfig, *,
                  normalize_quats: bool = False, sh: Tensor | None = None, sh_degree: int = 0,
                  campos: Tensor | None = None, need_active: bool = False,
                  metadata: bool = False) -> FusedProjection:
    """rade/projection.py:422-472 prepare, fused with rade/api.py:153-165's
    spherical_harmonics (sh (n,K,3) on means - campos) and
    splatting/metadata.py's prepare_metadata.  normalize_quats: quats are raw
    and normalised in-kernel with Torch's CUDA F.normalize bits."""
    pin = stages.Args()
    n = len(means)
    dev = means.device
    state = ProjectedGaussians(means.new_empty((n, 2)), means.new_empty((n, 4)),
                               torch.empty(n, dtype=torch.int32, device=dev),
                               torch.empty(n, dtype=torch.int32, device=dev),
                               means.new_empty(n), means.new_empty((n, 3)),
                               means.new_empty((n, 3)))
    colors = means.new_empty((n, 3)) if sh is not None else None
    active = (torch.empty((n, 3), dtype=torch.uint8, device=dev)
              if sh is not None and need_active else None)
    meta = (means.new_empty((n, 2)), means.new_empty(n), means.new_empty((n, 3))) \
        if metadata else (None, None, None)
    if n:
        check(lib.splat_rade_project_forward(
            n, pin(means), pin(quats), int(normalize_quats), pin(scales), pin(opacities),
            pin(view), pin(projection), pin(intrinsics), config.width, config.height,
            float(config.near), stages._far(config.far), float(config.radius_clip),
            float(config.kernel_size), ptr(state.centers), ptr(state.conics), ptr(state.radii),
            ptr(state.tile_counts), ptr(state.depths), ptr(state.ray_planes),
            ptr(state.normals), int(sh_degree), 0 if sh is None else sh.shape[1], pin(sh),
            pin(campos), ptr(colors), ptr(active), ptr(meta[0]), ptr(meta[1]), ptr(meta[2]),
            stages._stream(means)), "rade_project_forward")
    return FusedProjection(state, colors, active, *meta)


def prepare(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor, view: Tensor,
            projection: Tensor, intrinsics: Tensor, config: ViewConfig, *,
            normalize_quats: bool = False) -> ProjectedGaussians:
    """rade/projection.py:422-472 (quats normalised unless normalize_quats)."""
    return prepare_fused(means, quats, scales, opacities, view, projection, intrinsics, config,
                         normalize_quats=normalize_quats).state


def backward(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor, view: Tensor,
             projection: Tensor, intrinsics: Tensor, config: ViewConfig,
             state: ProjectedGaussians, grad_centers: Tensor | None,
             grad_conics: Tensor | None, grad_planes: Tensor | None,
             grad_normals: Tensor | None, needs: tuple[bool, ...], *,
             normalize_quats: bool = False, sh: Tensor | None = None, sh_degree: int = 0,
             campos: Tensor | None = None, active: Tensor | None = None,
             grad_colors: Tensor | None = None, need_sh: bool = False,
             need_campos: bool = False) -> list[Tensor | None]:
    """rade/projection.py:475-551 (+ the SH backward when sh is given):
    [means, quats, scales, opacities, view, projection, sh, campos]
    gradients (None where not needed)."""
    out: list[Tensor | None] = [None] * 8
    with_sh = sh is not None
    if not (any(needs) or (with_sh and (need_sh or need_campos))):
        return out
    pin = stages.Args()
    tensors = [means, quats, scales, opacities]
    grads = [torch.empty_like(t) if need else None for t, need in zip(tensors, needs[:4])]
    n = len(means)
    cam = means.new_zeros(32) if any(needs[4:6]) else None
    # the SH VJP runs whenever sh is given (its direction gradient feeds
    # means and the camera centre); coefficient gradients are kept if asked
    g_sh = torch.empty_like(sh) if with_sh else None
    g_campos = means.new_zeros(3) if with_sh and need_campos and campos is not None else None
    if n:
        check(lib.splat_rade_project_backward(
            n, pin(means), pin(quats), int(normalize_quats), pin(scales), pin(opacities),
            pin(view), pin(projection), pin(intrinsics), config.width, config.height,
            float(config.kernel_size), ptr(state.radii), pin(grad_centers), pin(grad_conics),
            pin(grad_planes), pin(grad_normals), *[ptr(g) for g in grads],
            ptr(None if cam is None else cam[:16]), ptr(None if cam is None else cam[16:]),
            int(sh_degree), 0 if sh is None else sh.shape[1], pin(sh), pin(campos), pin(active),
            pin(grad_colors), ptr(g_sh), ptr(g_campos), stages._stream(means)),
            "rade_project_backward")
    out[:4] = grads
    if needs[4]:
        out[4] = cam[:16].reshape(4, 4)
    if len(needs) > 5 and needs[5]:
        out[5] = cam[16:].reshape(4, 4)
    if with_sh and need_sh:
        out[6] = g_sh
    if g_campos is not None:
        out[7] = g_campos
    return out
