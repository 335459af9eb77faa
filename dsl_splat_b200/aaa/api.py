"""aaa.rasterize: AAA-Gaussians with OpenCV poses (aaa/api.py:1-221) on the
sm_100a kernels.

Same signature, validation, defaults (AAA's recommended settings), batching,
metadata and result type as the reference.  Per call: the cameras are
lowered with Torch (aaa/cameras.py), every view is preprocessed (adaptive 3D
filter, EWA compensation, culling), all views are binned with one host read
of their pair counts, and each view is blended by the HIER kernel inside one
autograd Function.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from numbers import Integral
from typing import Any, Sequence

import torch
from torch import Tensor

from ..cameras import validate_camera_options
from ..inputs import batch_item, normalize_inputs, spherical_harmonics
from ..statistics import StatisticsRequest, prepare_statistics
from ..training import prepare_training_metadata
from . import stages
from .autograd import RasterizeView
from .cameras import prepare_cameras
from .config import default_settings, validate_settings
from .settings import ExtendedSettings


@dataclass(slots=True)
class RasterizationResult:
    """features (..., C, H, W, D), alpha (..., C, H, W, 1) (aaa/api.py:23-44)."""

    features: Tensor
    alpha: Tensor
    meta: dict[str, Any]
    statistics: dict[str, Tensor] = field(default_factory=dict)

    @property
    def radii(self) -> Tensor:
        return self.meta["radii"]

    @property
    def means2d(self) -> Tensor:
        return self.meta["means2d"]

    @property
    def extra_features(self) -> Tensor | None:
        return self.meta.get("render_extra_signals")


def _check_arguments(features, sh_coeffs, sh_degree):
    if (features is None) == (sh_coeffs is None):
        raise ValueError("provide exactly one of features or sh_coeffs")
    if sh_coeffs is not None and (not isinstance(sh_coeffs, Tensor) or sh_coeffs.ndim < 3):
        raise ValueError("sh_coeffs must have shape (...,N,K,3) or (...,C,N,K,3)")
    if sh_coeffs is not None and sh_degree is None:
        sh_degree = min(3, math.isqrt(sh_coeffs.shape[-2]) - 1)
    if features is not None and sh_degree is not None:
        raise ValueError("sh_degree requires sh_coeffs")
    if sh_degree is not None and (isinstance(sh_degree, bool) or not isinstance(sh_degree, Integral)
                                  or sh_degree not in range(4)):
        raise ValueError("sh_degree must be an integer in [0,3]")
    return sh_degree


@torch.no_grad()
def _dense_geometry(frames, states, layout) -> dict[str, Tensor]:
    """aaa/metadata.py:55-91 _geometry: per view the pixel projection of the
    means (densification statistics only), radii = ceil of the bounding half
    extents, effective opacities and tile counts; zero for culled rows (one
    kernel per view, stages.metadata)."""
    views, n, dev = len(frames), layout.n, layout.device
    radii = torch.empty((views, n, 2), device=dev, dtype=torch.int32)
    means2d = torch.empty((views, n, 2), device=dev, dtype=torch.float32)
    opacities = torch.empty((views, n), device=dev, dtype=torch.float32)
    for v, ((b, c, view, _features, _bg), st) in enumerate(zip(frames, states)):
        vm = batch_item(batch_item(layout.viewmats, b), c)
        focal = (view.width / (2 * view.tanfovx), view.height / (2 * view.tanfovy))
        stages.metadata(vm, focal, view.principal, layout.means[b], st, radii[v], means2d[v],
                        opacities[v])
    tiles = torch.stack([st.tiles for st in states]) if states else torch.empty(
        (0, n), device=dev, dtype=torch.int32)
    shape = (layout.batch_count, layout.cameras, n)
    return {"radii": radii.reshape(shape + (2,)), "means2d": means2d.reshape(shape + (2,)),
            "opacities": opacities.reshape(shape), "tiles_per_gauss": tiles.reshape(shape)}


def rasterize(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor, viewmats: Tensor,
              Ks: Tensor, width: int, height: int, *, features: Tensor | None = None,
              sh_coeffs: Tensor | None = None, sh_degree: int | None = None,
              backgrounds: Tensor | None = None, extra_features: Tensor | None = None,
              filter3d: Tensor | None = None, near_plane: float = 0.01, far_plane: float = 1e10,
              radius_clip: float = 0.0, packed: bool = False, absgrad: bool = False,
              settings: ExtendedSettings | None = None,
              statistics: Sequence[StatisticsRequest] = ()) -> RasterizationResult:
    """Render AAA Gaussians with OpenCV world-to-camera poses and zero-skew K.

    Pass features (...,N,D) / (...,C,N,D), or SH coefficients (...,N,K,3) /
    (...,C,N,K,3).  Scales and opacities are activated; quaternions (wxyz)
    are normalised differentiably.  Defaults: AAA's antialiased HIER 64/8/4
    configuration.  First-order gradients reach the Gaussian parameters,
    features/SH, extras and poses; K, background and filter gradients are
    not supported (as in the reference)."""
    validate_camera_options(width, height, near_plane, far_plane, radius_clip)
    sh_degree = _check_arguments(features, sh_coeffs, sh_degree)
    # the raw quaternions go to the kernels, which normalise them with
    # F.normalize's bits and return their gradient (inputs.py:252)
    layout = normalize_inputs(means, quats, scales, opacities,
                              features if sh_coeffs is None else sh_coeffs, viewmats, Ks,
                              backgrounds, extra_features, filter3d, sh_degree,
                              normalize_quats=False)
    if settings is not None:
        validate_settings(settings)
    config = default_settings() if settings is None else settings.copy()
    stages.require_supported(config)
    cameras = prepare_cameras(layout.viewmats, layout.Ks, width, height, near_plane, far_plane)
    prepared_stats, statistics_outputs = (
        prepare_statistics(statistics, batch_dims=layout.batch_dims,
                           batch_count=layout.batch_count, cameras=layout.cameras, n=layout.n,
                           width=width, height=height, device=layout.device)
        if statistics else ([], {}))
    colors = layout.colors
    ones = torch.ones(layout.n, 1, device=layout.device, dtype=torch.float32)
    frames, states = [], []
    for b in range(layout.batch_count):
        bm = layout.means[b]
        for c in range(layout.cameras):
            value = colors.at(b, c)
            if sh_degree is not None:
                value = spherical_harmonics(value, bm - cameras.centers[b, c], sh_degree)
            parts = [value]
            if layout.extras is not None:
                parts.append(layout.extras.at(b, c))
            parts.append(ones)
            feats = torch.cat(parts, dim=-1)
            bg = torch.zeros(feats.shape[-1], device=layout.device, dtype=torch.float32)
            if layout.backgrounds is not None:
                bg[: colors.channels] = layout.backgrounds[b, c]
            view = cameras.view(b, c)
            filters = None if layout.filters is None else layout.filters[b]
            states.append(stages.preprocess(
                stages.AaaView(view.width, view.height, view.tanfovx, view.tanfovy,
                               view.principal, view.viewmatrix.detach(),
                               view.projmatrix.detach(), view.campos.detach()),
                config, bm.detach(), layout.quats[b].detach(), layout.scales[b].detach(),
                layout.opacities[b].detach(), None if filters is None else filters.detach(),
                radius_clip, raw_quats=True))
            frames.append((b, c, view, feats, bg))
    dense = _dense_geometry(frames, states, layout)
    # packed metadata keeps the rows whose rounded extents are positive
    # (training.py:27-34 on the dense radii); their per-view counts are read
    # in the binning's host synchronisation
    visible = ([m.sum() for m in (dense["radii"] > 0).all(-1).reshape(-1, layout.n)]
               if packed else [])
    bins, visible_counts = stages.bin_and_sort_many(states, width, height, host_reads=visible)
    training = prepare_training_metadata(dense, layout, packed=packed, absgrad=absgrad,
                                         visible_counts=visible_counts if packed else None)
    meta = training.values
    meta.update(width=width, height=height, tile_size=16, tile_width=(width + 15) // 16,
                tile_height=(height + 15) // 16, n_cameras=layout.cameras, packed=packed,
                backend="aaa-b200", with_eval3d=True, conics=None, supports_means2d_grad=True,
                screen_gradient_mode="rigid_footprint_translation")
    grad_enabled = torch.is_grad_enabled()
    channels = colors.channels
    outputs, alphas, extras = [], [], []
    for i, ((b, c, view, feats, bg), st) in enumerate(zip(frames, states)):
        screen = None if training.screen is None else training.screen[b, c]
        filters = None if layout.filters is None else layout.filters[b].detach()
        image, _, _ = RasterizeView.apply(
            layout.means[b], layout.quats[b], layout.scales[b], layout.opacities[b], feats,
            screen, view.viewmatrix, view.projmatrix, view.campos,
            stages.AaaView(view.width, view.height, view.tanfovx, view.tanfovy, view.principal,
                           view.viewmatrix.detach(), view.projmatrix.detach(),
                           view.campos.detach()),
            config, st, bins[i], bg, filters, training.absolute_targets[i], grad_enabled,
            prepared_stats[i] if statistics else None)
        hwc = image.permute(1, 2, 0)
        if layout.n == 0:
            hwc = hwc + bg
        outputs.append(hwc[..., :channels])
        alphas.append(hwc[..., -1:])
        if layout.extras is not None:
            extras.append(hwc[..., channels:-1])
    shape = layout.batch_dims + (layout.cameras, height, width)
    if extras:
        meta["render_extra_signals"] = torch.stack(extras).reshape(
            shape + (layout.extras.channels,))
    return RasterizationResult(torch.stack(outputs).reshape(shape + (channels,)),
                               torch.stack(alphas).reshape(shape + (1,)), meta,
                               statistics_outputs)


__all__ = ["rasterize", "RasterizationResult", "ExtendedSettings", "default_settings"]
