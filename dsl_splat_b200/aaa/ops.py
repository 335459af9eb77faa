"""aaa.ops: composable, differentiable AAA stages for one OpenCV camera
(aaa/ops.py:1-464) on the sm_100a kernels.

* prepare_gaussians: the preprocessing and the remainder cull of one view
  (the kernels normalise the raw quaternions); its backward is the
  preprocessing adjoint for the Gaussians and the camera adjoint for the
  pose.
* bin_and_sort: key emission, the stable sort and the tile ranges.
* rasterize_to_pixels: the HIER 64/8/4 blend of (N,D) features plus alpha
  over reused geometry and tiles; its backward reads the blend records.

Same public names, result types, argument checks and error messages as the
reference; aaa.rasterize keeps its own single autograd Function.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Sequence

import torch
from torch import Tensor
from torch.autograd.function import once_differentiable

from ..cameras import PinholeCamera, validate_camera_options
from ..inputs import check_tensor, spherical_harmonics
from ..statistics import StatisticsRequest, prepare_statistics
from . import stages
from .cameras import prepare_cameras
from .config import default_settings, validate_settings
from .settings import ExtendedSettings

__all__ = ["prepare_gaussians", "bin_and_sort", "rasterize_to_pixels", "spherical_harmonics",
           "GaussianGeometry", "GaussianTiles", "PixelResult"]


@dataclass(slots=True)
class GaussianGeometry:
    """AAA ray transforms and bounds; rejected rows are identified by radii=0.

    ray_transforms (N,4,4) and opacities (N) are differentiable; bounds,
    visibility and tile membership are discrete and fixed in the backward.
    Bounding centres are not gsplat's projected-centre metadata.
    """

    ray_transforms: Tensor
    opacities: Tensor
    radii: Tensor
    bounding_centers: Tensor
    half_extents: Tensor
    tiles_touched: Tensor
    valid: Tensor
    depths: Tensor
    _view: stages.AaaView = field(repr=False)
    _settings: ExtendedSettings = field(repr=False)

    def _state(self) -> stages.AaaState:
        return stages.AaaState(self.bounding_centers, self.half_extents, self.depths,
                               self.ray_transforms.detach(), self.opacities.detach(), self.radii,
                               self.tiles_touched, self.valid)


@dataclass(slots=True)
class GaussianTiles:
    ranges: Tensor
    gaussian_ids: Tensor
    _geometry: GaussianGeometry = field(repr=False)
    _bins: dict = field(repr=False)


@dataclass(slots=True)
class PixelResult:
    """Owned (H,W,D) features and differentiable (H,W,1) alpha."""

    features: Tensor
    alpha: Tensor
    statistics: dict[str, Tensor] = field(default_factory=dict)


class _PrepareGaussians(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, means, quats, scales, opacities, filters, viewmatrix, projmatrix,
                campos, view: stages.AaaView, settings: ExtendedSettings, radius_clip: float,
                grad_enabled: bool):
        st = stages.preprocess(view, settings, means.detach(), quats.detach(), scales.detach(),
                               opacities.detach(),
                               None if filters is None else filters.detach(), radius_clip,
                               raw_quats=True)
        outputs = (st.transforms, st.opacity, st.radii, st.centers, st.rects, st.tiles,
                   st.valid, st.depths)
        ctx.mark_non_differentiable(*outputs[2:])
        ctx.set_materialize_grads(False)
        if grad_enabled and any(ctx.needs_input_grad[:8]):
            ctx.save_for_backward(means, quats, scales, opacities, filters)
            ctx.view, ctx.settings, ctx.state = view, settings, st
        return outputs

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, grad_transform, grad_opacity, *unused):
        none = (None,) * 12
        if grad_transform is None and grad_opacity is None:
            return none
        means, quats, scales, opacities, filters = ctx.saved_tensors
        st = ctx.state
        # the adjoints take the transform gradient in the blend backward's
        # (transposed) layout
        up_t = (torch.zeros_like(st.transforms) if grad_transform is None
                else grad_transform.transpose(-1, -2).contiguous())
        up_o = (torch.zeros_like(st.opacity) if grad_opacity is None
                else grad_opacity.contiguous())
        needs = ctx.needs_input_grad
        g_means = g_quats = g_scales = g_opac = None
        if any(needs[:4]):
            g_opac, g_means, g_scales, g_quats = stages.preprocess_backward(
                ctx.view, ctx.settings, means, quats, scales, opacities, st, up_t, up_o)
        g_view = g_proj = g_campos = None
        if any(needs[5:8]):
            g_view, g_proj, g_campos = stages.camera_backward(
                ctx.view, ctx.settings, means, quats, scales, filters, st, up_t, up_o)
        return (g_means if needs[0] else None, g_quats if needs[1] else None,
                g_scales if needs[2] else None,
                g_opac.reshape_as(opacities) if needs[3] else None,
                None,  # the 3D filter is a constant, as in AAA
                g_view if needs[5] else None, g_proj if needs[6] else None,
                g_campos if needs[7] else None, None, None, None, None)


class _RasterizePixels(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, transforms, opacity, features, geometry: GaussianGeometry,
                tiles: GaussianTiles, background, cull: bool, grad_enabled: bool, statistics):
        st = stages.AaaState(None, None, None, transforms.detach().contiguous(),
                             opacity.detach().contiguous(), geometry.radii, None, None)
        features = features.contiguous()
        needs_backward = grad_enabled and any(ctx.needs_input_grad[:3])
        view = geometry._view
        image, final_t, _, records = stages.render(
            st, tiles._bins, features.detach(), background, view.width, view.height, cull,
            record_capacity=stages.RECORD_CAPACITY if needs_backward else 0,
            statistics=statistics)
        ctx.set_materialize_grads(False)
        if needs_backward:
            ctx.save_for_backward(features, image, final_t, background)
            ctx.state, ctx.bins, ctx.records, ctx.cull = st, tiles._bins, records, cull
            ctx.size = (view.width, view.height)
        return image

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, grad_color):
        none = (None,) * 9
        if grad_color is None:
            return none
        features, image, final_t, background = ctx.saved_tensors
        W, H = ctx.size
        g_tr, g_op, g_col, _, _ = stages.render_backward(
            ctx.state, ctx.bins, features, background, image, final_t, grad_color.contiguous(),
            W, H, ctx.cull, records=ctx.records)
        needs = ctx.needs_input_grad
        return (g_tr.transpose(-1, -2) if needs[0] else None, g_op if needs[1] else None,
                g_col if needs[2] else None) + (None,) * 6


def prepare_gaussians(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor,
                      camera: PinholeCamera, *, filter3d: Tensor | None = None,
                      radius_clip: float = 0.0,
                      settings: ExtendedSettings | None = None) -> GaussianGeometry:
    """Prepare one view without features; supports Gaussian and pose gradients.

    Inputs are CUDA float32, shapes (N,3), (N,4), (N,3), (N,).  Quaternion
    normalisation is differentiable.  Reuse requires unchanged camera,
    geometry, opacity, filtering and settings.  Culling and bounds are not
    differentiated."""
    if (not isinstance(means, Tensor) or not means.is_cuda or means.ndim != 2
            or means.shape[1] != 3):
        raise ValueError("means must be CUDA float32 (N,3)")
    n, device = len(means), means.device
    for name, value, shape in (("means", means, (n, 3)), ("quats", quats, (n, 4)),
                               ("scales", scales, (n, 3)), ("opacities", opacities, (n,))):
        check_tensor(name, value, device, shape)
    if filter3d is not None:
        check_tensor("filter3d", filter3d, device)
        if filter3d.shape not in ((n,), (n, 1)):
            raise ValueError("filter3d must have shape (N,) or (N,1)")
    if camera.viewmat.device != device:
        raise ValueError("camera and Gaussians must be on the same device")
    if radius_clip < 0 or not math.isfinite(radius_clip):
        raise ValueError("radius_clip must be finite and nonnegative")
    if settings is not None:
        validate_settings(settings)
    options = default_settings() if settings is None else settings.copy()
    stages.require_supported(options)
    validate_camera_options(camera.width, camera.height, camera.near_plane, camera.far_plane, 0.0)
    check_tensor("viewmat", camera.viewmat, device, (4, 4))
    check_tensor("K", camera.K, device, (3, 3))
    if torch.is_grad_enabled() and camera.K.requires_grad:
        raise NotImplementedError("intrinsics gradients are not supported")
    lowered = prepare_cameras(camera.viewmat[None, None], camera.K.detach()[None, None],
                              camera.width, camera.height, camera.near_plane,
                              camera.far_plane).view(0, 0)
    view = stages.AaaView(lowered.width, lowered.height, lowered.tanfovx, lowered.tanfovy,
                          lowered.principal, lowered.viewmatrix.detach(),
                          lowered.projmatrix.detach(), lowered.campos.detach())
    filters = None if filter3d is None else filter3d.reshape(n)
    values = _PrepareGaussians.apply(means, quats, scales, opacities, filters,
                                     lowered.viewmatrix, lowered.projmatrix, lowered.campos,
                                     view, options, float(radius_clip), torch.is_grad_enabled())
    return GaussianGeometry(*values, _view=view, _settings=options)


@torch.no_grad()
def bin_and_sort(geometry: GaussianGeometry) -> GaussianTiles:
    """Build AAA tile intersections and keys using its configured depth order."""
    view = geometry._view
    bins, _ = stages.bin_and_sort_many([geometry._state()], view.width, view.height)
    return GaussianTiles(bins[0]["ranges"], bins[0]["point_list"], geometry, bins[0])


def rasterize_to_pixels(geometry: GaussianGeometry, tiles: GaussianTiles, features: Tensor,
                        background: Tensor | None = None, *,
                        statistics: Sequence[StatisticsRequest] = ()) -> PixelResult:
    """Blend (N,D) attributes and alpha, reusing geometry and sorted tiles.

    Features can be signed and have any positive channel count.  Background is
    constant; its gradient is unsupported.  Rendering follows AAA HIER 64/8/4."""
    if tiles._geometry is not geometry:
        raise ValueError("tiles must have been built from this geometry")
    device, n = geometry.radii.device, len(geometry.radii)
    check_tensor("features", features, device)
    if features.ndim != 2 or features.shape[0] != n or features.shape[1] <= 0:
        raise ValueError("features must have shape (N,D), D > 0")
    channels = features.shape[1]
    if background is not None:
        check_tensor("background", background, device, (channels,))
        if torch.is_grad_enabled() and background.requires_grad:
            raise NotImplementedError("background gradients are not supported")
    attributes = torch.cat((features, features.new_ones(n, 1)), -1)
    bg = features.new_zeros(channels + 1)
    if background is not None:
        bg[:channels] = background.detach()
    view = geometry._view
    prepared, outputs = (
        prepare_statistics(statistics, batch_dims=(), batch_count=1, cameras=1, n=n,
                           width=view.width, height=view.height, device=device)
        if statistics else ([], {}))
    cull = bool(geometry._settings.culling_settings.hierarchical_4x4_culling)
    color = _RasterizePixels.apply(geometry.ray_transforms, geometry.opacities, attributes,
                                   geometry, tiles, bg, cull, torch.is_grad_enabled(),
                                   prepared[0] if statistics else None).permute(1, 2, 0)
    return PixelResult(color[..., :channels], color[..., -1:],
                       {name: value[0] for name, value in outputs.items()})
