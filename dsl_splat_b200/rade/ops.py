"""Differentiable single-view RaDe-GS stages (rade/ops.py:1-380):
prepare_gaussians -> bin_and_sort -> rasterize_to_pixels, for callers that
reuse geometry or compose rendering stages."""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Sequence

import torch
from torch import Tensor

from .. import stages
from ..camera_prep import prepare_camera
from ..cameras import PinholeCamera
from ..inputs import check_tensor, spherical_harmonics
from ..statistics import StatisticsRequest, prepare_statistics
from .autograd import Project, Render
from .projection import ProjectedGaussians, ViewConfig


@dataclass(slots=True)
class GaussianGeometry:
    """Only rows with radii>0 define centers and conics; bounds are discrete."""

    centers: Tensor
    conics: Tensor
    radii: Tensor
    tile_counts: Tensor
    depths: Tensor
    ray_planes: Tensor
    normals: Tensor
    _intrinsics: Tensor = field(repr=False)
    _config: ViewConfig = field(repr=False)

    def _state(self) -> ProjectedGaussians:
        return ProjectedGaussians(self.centers, self.conics, self.radii, self.tile_counts,
                                  self.depths, self.ray_planes, self.normals)


@dataclass(slots=True)
class GaussianTiles:
    ranges: Tensor
    gaussian_ids: Tensor
    _geometry: GaussianGeometry = field(repr=False)


@dataclass(slots=True)
class PixelResult:
    features: Tensor
    alpha: Tensor
    depth: Tensor
    median_depth: Tensor
    normals: Tensor
    statistics: dict[str, Tensor] = field(default_factory=dict)


def prepare_gaussians(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor,
                      camera: PinholeCamera, *, radius_clip: float = 0.0,
                      kernel_size: float = 0.0) -> GaussianGeometry:
    """rade/ops.py:245-299."""
    if not isinstance(means, Tensor) or not means.is_cuda or means.ndim != 2 or means.shape[1] != 3:
        raise ValueError("means must be CUDA float32 (N,3)")
    n, device = len(means), means.device
    for name, value, shape in (("means", means, (n, 3)), ("quats", quats, (n, 4)),
                               ("scales", scales, (n, 3)), ("opacities", opacities, (n,))):
        check_tensor(name, value, device, shape)
    view, full, intrinsics, config = prepare_camera(camera, radius_clip)
    if view.device != device:
        raise ValueError("camera and Gaussians must use the same CUDA device")
    if not math.isfinite(kernel_size) or kernel_size < 0:
        raise ValueError("kernel_size must be finite and nonnegative")
    config = ViewConfig(config.width, config.height, config.near, config.far,
                        config.radius_clip, "radius", float(kernel_size))
    # quats are normalised in-kernel (Torch's F.normalize bits, with its VJP)
    ctr, con, _, radii, tiles, depths, planes, normals, *_ = Project.apply(
        means.contiguous(), quats.contiguous(), scales.contiguous(), opacities.contiguous(),
        None, view, full, None, intrinsics, config, None, torch.is_grad_enabled())
    return GaussianGeometry(ctr, con, radii, tiles, depths, planes, normals, intrinsics, config)


def bin_and_sort(geometry: GaussianGeometry) -> GaussianTiles:
    """rade/ops.py:302-312 (radial sort distances)."""
    cfg = geometry._config
    bins = stages.bin_and_sort(geometry._state(), cfg.width, cfg.height)
    tiles = GaussianTiles(bins["ranges"], bins["point_list"], geometry)
    return tiles


def rasterize_to_pixels(geometry: GaussianGeometry, tiles: GaussianTiles, features: Tensor,
                        background: Tensor | None = None, *,
                        statistics: Sequence[StatisticsRequest] = ()) -> PixelResult:
    """rade/ops.py:315-369."""
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
    cfg = geometry._config
    prepared, outputs = (prepare_statistics(statistics, batch_dims=(), batch_count=1, cameras=1,
                                            n=n, width=cfg.width, height=cfg.height,
                                            device=device)
                         if statistics else ([], {}))
    bg = features.new_zeros(channels) if background is None else background.contiguous()
    bins = dict(ranges=tiles.ranges, point_list=tiles.gaussian_ids)
    feats, _, *geometry_images = Render.apply(
        geometry.centers, geometry.conics, geometry.ray_planes, geometry.normals, features, None,
        None, bg, bins, geometry._intrinsics, cfg, None, None,
        prepared[0] if statistics else None, torch.is_grad_enabled())
    images = (feats, *geometry_images)
    return PixelResult(*images, {name: value[0] for name, value in outputs.items()})


__all__ = ["prepare_gaussians", "bin_and_sort", "rasterize_to_pixels", "spherical_harmonics",
           "GaussianGeometry", "GaussianTiles", "PixelResult"]
