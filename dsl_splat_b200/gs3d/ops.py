"""Composable differentiable gs3d stages (gs3d/ops.py:1-338).

prepare_gaussians -> bin_and_sort -> rasterize_to_pixels, each an autograd
Function over the sm_100a kernels, for callers that reuse geometry or render
several attribute sets from one binning.
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace
from typing import Any, Sequence

import torch
from torch import Tensor
from torch.autograd.function import once_differentiable
from torch.nn.functional import normalize

from .. import stages
from ..camera_prep import ViewConfig, prepare_camera
from ..cameras import PinholeCamera
from ..inputs import check_tensor, spherical_harmonics
from ..statistics import PreparedStatistics, StatisticsRequest, prepare_statistics
from .api import validate_tile_mode


@dataclass(slots=True)
class GaussianGeometry:
    """Only rows with radii>0 define centers and conics; bounds are discrete."""

    centers: Tensor
    conics: Tensor
    radii: Tensor
    tile_counts: Tensor
    depths: Tensor
    _config: ViewConfig = field(repr=False)

    def _state(self) -> stages.ProjectedGaussians:
        return stages.ProjectedGaussians(self.centers, self.conics, self.radii,
                                         self.tile_counts, self.depths)


@dataclass(slots=True)
class GaussianTiles:
    ranges: Tensor
    gaussian_ids: Tensor
    _geometry: GaussianGeometry = field(repr=False)


@dataclass(slots=True)
class PixelResult:
    features: Tensor
    alpha: Tensor
    statistics: dict[str, Tensor] = field(default_factory=dict)


class _Project(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, means, quats, scales, opacities, view, full, intrinsics,
                config: ViewConfig, grad_enabled: bool):
        st = stages.project(means, quats, scales, opacities, view, full, intrinsics, config.width,
                            config.height, config.near, config.far, config.radius_clip,
                            config.tile_mode)
        if grad_enabled and any(ctx.needs_input_grad[:6]):
            ctx.save_for_backward(means, quats, scales, opacities, view, full, intrinsics,
                                  st.centers, st.conics, st.radii, st.tile_counts, st.depths)
            ctx.config = config
        ctx.mark_non_differentiable(st.radii, st.tile_counts, st.depths)
        ctx.set_materialize_grads(False)
        return st.centers, st.conics, st.radii, st.tile_counts, st.depths

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, centers: Tensor | None, conics: Tensor | None, *unused):
        if centers is None and conics is None:
            return (None,) * 9
        values = ctx.saved_tensors
        state = stages.ProjectedGaussians(*values[7:])
        cfg = ctx.config
        grads = stages.project_backward(
            *values[:7], cfg.width, cfg.height, state,
            torch.zeros_like(state.centers) if centers is None else centers.contiguous(),
            torch.zeros_like(state.conics) if conics is None else conics.contiguous(),
            tuple(ctx.needs_input_grad[:6]))
        return (*grads, None, None, None)


class _Pixels(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, centers, conics, features, ranges, ids, background,
                config: ViewConfig, statistics: PreparedStatistics | None, grad_enabled: bool):
        out = stages.render(stages.ProjectedFootprint(centers, conics),
                            dict(ranges=ranges, point_list=ids), features, None, True, background,
                            config.width, config.height, statistics=statistics)
        if grad_enabled and any(ctx.needs_input_grad[:3]):
            ctx.save_for_backward(centers, conics, features, ranges, ids, background,
                                  out.transmittance, out.contributors)
            ctx.config = config
        ctx.set_materialize_grads(False)
        return out.features

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, gradient: Tensor | None):
        if gradient is None:
            return (None,) * 9
        centers, conics, features, ranges, ids, background, final_t, contrib = ctx.saved_tensors
        cfg = ctx.config
        gc, gq, gf, _, _ = stages.render_backward(
            stages.ProjectedFootprint(centers, conics), dict(ranges=ranges, point_list=ids),
            features, None, True, background, final_t, contrib, gradient, cfg.width, cfg.height,
            constant_tail=1, need_a=ctx.needs_input_grad[2])
        needs = ctx.needs_input_grad
        return (gc if needs[0] else None, gq if needs[1] else None, gf if needs[2] else None,
                None, None, None, None, None, None)


def prepare_gaussians(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor,
                      camera: PinholeCamera, *, radius_clip: float = 0.0,
                      tile_mode: str = "radius") -> GaussianGeometry:
    """gs3d/ops.py:215-259."""
    if not isinstance(means, Tensor) or not means.is_cuda or means.ndim != 2 or means.shape[1] != 3:
        raise ValueError("means must be CUDA float32 (N,3)")
    validate_tile_mode(tile_mode)
    n, device = len(means), means.device
    for name, value, shape in (("means", means, (n, 3)), ("quats", quats, (n, 4)),
                               ("scales", scales, (n, 3)), ("opacities", opacities, (n,))):
        check_tensor(name, value, device, shape)
    view, full, intrinsics, config = prepare_camera(camera, radius_clip)
    if view.device != device:
        raise ValueError("camera and Gaussians must use the same CUDA device")
    config = replace(config, tile_mode=tile_mode)
    out = _Project.apply(means.contiguous(), normalize(quats, dim=-1).contiguous(),
                         scales.contiguous(), opacities.contiguous(), view, full, intrinsics,
                         config, torch.is_grad_enabled())
    return GaussianGeometry(*out, config)


def bin_and_sort(geometry: GaussianGeometry) -> GaussianTiles:
    """gs3d/ops.py:262-270."""
    bins = stages.bin_and_sort(geometry._state(), geometry._config.width, geometry._config.height,
                               tile_mode=geometry._config.tile_mode)
    return GaussianTiles(bins["ranges"], bins["point_list"], geometry)


def rasterize_to_pixels(geometry: GaussianGeometry, tiles: GaussianTiles, features: Tensor,
                        background: Tensor | None = None, *,
                        statistics: Sequence[StatisticsRequest] = ()) -> PixelResult:
    """gs3d/ops.py:273-327."""
    if tiles._geometry is not geometry:
        raise ValueError("tiles must have been built from this geometry")
    n, device = len(geometry.radii), geometry.radii.device
    check_tensor("features", features, device)
    if features.ndim != 2 or features.shape[0] != n or features.shape[1] <= 0:
        raise ValueError("features must have shape (N,D), D>0")
    channels = features.shape[1]
    if background is not None:
        check_tensor("background", background, device, (channels,))
        if torch.is_grad_enabled() and background.requires_grad:
            raise NotImplementedError("background gradients are not supported")
    bg = features.new_zeros(channels + 1)
    if background is not None:
        bg[:channels] = background
    cfg = geometry._config
    prepared, outputs = (prepare_statistics(statistics, batch_dims=(), batch_count=1, cameras=1,
                                            n=n, width=cfg.width, height=cfg.height,
                                            device=device)
                         if statistics else ([], {}))
    image = _Pixels.apply(geometry.centers, geometry.conics, features, tiles.ranges,
                          tiles.gaussian_ids, bg, cfg, prepared[0] if statistics else None,
                          torch.is_grad_enabled())
    return PixelResult(image[..., :channels], image[..., -1:],
                       {name: value[0] for name, value in outputs.items()})


__all__ = ["prepare_gaussians", "bin_and_sort", "rasterize_to_pixels", "spherical_harmonics",
           "GaussianGeometry", "GaussianTiles", "PixelResult"]
