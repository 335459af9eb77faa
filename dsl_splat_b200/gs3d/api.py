"""Original 3DGS entry point (gs3d/api.py:1-265) on the sm_100a kernels.

Same signature, validation, batching, metadata and result type as the
reference; the per-view work runs as: one camera launch for all views, one
fused projection+SH+metadata launch per view, binning of all views with a
single host read of their pair counts, and one blend launch per view.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from numbers import Integral
from typing import Any, Sequence

import torch
from torch import Tensor

from ..camera_prep import ViewConfig, prepare_cameras, prepare_cameras_with_centers
from ..cameras import validate_camera_options
from ..inputs import batch_item, normalize_inputs
from ..statistics import StatisticsRequest, prepare_statistics
from ..training import prepare_training_metadata
from .. import stages
from .autograd import ProjectView, ProjectViews, RenderView

TILE_MODES = ("radius", "snugbox", "accutile")


def validate_tile_mode(mode) -> None:
    """splatting/intersections.py:24-26."""
    if mode not in TILE_MODES:
        raise ValueError("tile_mode must be 'radius', 'snugbox' or 'accutile'")


@dataclass(slots=True)
class RasterizationResult:
    """Channel-last images and training metadata (gs3d/api.py:25-44)."""

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


def _check_sh(sh_coeffs, sh_degree, features):
    if (features is None) == (sh_coeffs is None):
        raise ValueError("provide exactly one of features or sh_coeffs")
    if sh_coeffs is not None:
        if not isinstance(sh_coeffs, Tensor) or sh_coeffs.ndim < 3:
            raise ValueError("sh_coeffs must have shape (...,N,K,3) or (...,C,N,K,3)")
        if sh_degree is None:
            sh_degree = min(3, math.isqrt(sh_coeffs.shape[-2]) - 1)
    elif sh_degree is not None:
        raise ValueError("sh_degree requires sh_coeffs")
    if sh_degree is not None and (isinstance(sh_degree, bool) or not isinstance(sh_degree, Integral)
                                  or sh_degree not in range(4)):
        raise ValueError("sh_degree must be an integer in [0,3]")
    return sh_degree


_ZERO_BACKGROUNDS: dict = {}


def _zero_background(device: torch.device, channels: int) -> Tensor:
    """A zero background vector, made once per device and size (the kernels
    only read it)."""
    key = (device, channels)
    bg = _ZERO_BACKGROUNDS.get(key)
    if bg is None:
        bg = _ZERO_BACKGROUNDS[key] = torch.zeros(channels, device=device)
    return bg


def rasterize(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor, viewmats: Tensor,
              Ks: Tensor, width: int, height: int, *, features: Tensor | None = None,
              sh_coeffs: Tensor | None = None, sh_degree: int | None = None,
              backgrounds: Tensor | None = None, extra_features: Tensor | None = None,
              near_plane: float = 0.2, far_plane: float = math.inf, radius_clip: float = 0.0,
              packed: bool = False, absgrad: bool = False,
              statistics: Sequence[StatisticsRequest] = (),
              tile_mode: str = "radius") -> RasterizationResult:
    """Render original 3DGS (centre-depth order, square tile bounds).

    Inputs are activated scales/opacities and wxyz quaternions (normalised
    here).  means2d is in CUDA raster coordinates (integer pixel centres,
    K-projected position minus 0.5), zero for culled rows.  Gradients reach
    means, quats, scales, opacities, features/SH, extras and viewmats.
    """
    validate_tile_mode(tile_mode)
    validate_camera_options(width, height, near_plane, far_plane, radius_clip)
    sh_degree = _check_sh(sh_coeffs, sh_degree, features)
    # Quaternions reach the projection kernels raw: they apply inputs.py:252's
    # F.normalize with Torch's CUDA bits and its VJP in the backward.
    layout = normalize_inputs(means, quats, scales, opacities,
                              features if sh_coeffs is None else sh_coeffs, viewmats, Ks,
                              backgrounds, extra_features, None, sh_degree,
                              normalize_quats=False)
    with_centers = sh_degree is not None and sh_degree > 0
    # Camera status codes are read in the same host synchronisation as the
    # pair counts below (one read per call instead of two).
    camera_status: list = []
    if with_centers:
        full, centers = prepare_cameras_with_centers(layout.viewmats, layout.Ks, width, height,
                                                     camera_status)
    else:
        full = prepare_cameras(layout.viewmats, layout.Ks, width, height, camera_status)
        centers = None
    config = ViewConfig(width, height, near_plane, far_plane, radius_clip, tile_mode)
    grad_enabled = torch.is_grad_enabled()
    frames = []
    # per batch: (cameras, n, ...) stacks of the dense metadata
    dense: dict[str, list[Tensor]] = {k: [] for k in ("radii", "means2d", "opacities",
                                                      "tiles_per_gauss", "conics")}
    for b in range(layout.batch_count):
        bm, bq = layout.means[b], layout.quats[b]
        bs, bo = layout.scales[b], layout.opacities[b]
        shared_sh = sh_degree is not None and not layout.colors.per_view
        if layout.cameras > 1 and (sh_degree is None or shared_sh):
            # every camera of the batch in one projection launch each way
            C = layout.cameras
            out = ProjectViews.apply(
                bm, bq, bs, bo, layout.colors.at(b, 0) if sh_degree is not None else None,
                batch_item(layout.viewmats, b), batch_item(full, b),
                batch_item(centers, b) if with_centers else None, batch_item(layout.Ks, b),
                config, sh_degree, grad_enabled)
            radii, tiles, depths, m2d, mop, mcon = out[3 * C:]
            for c in range(C):
                ctr, con, col = out[c], out[C + c], out[2 * C + c]
                colors = col if sh_degree is not None else layout.colors.at(b, c)
                extras = None if layout.extras is None else layout.extras.at(b, c)
                bg = (None if layout.backgrounds is None
                      else batch_item(batch_item(layout.backgrounds, b), c))
                frames.append((b, c, ctr, con, colors, extras, bg,
                               stages.ProjectedGaussians(ctr, con, radii[c], tiles[c],
                                                         depths[c])))
            dense["radii"].append(radii[..., None].expand(-1, -1, 2))
            dense["means2d"].append(m2d)
            dense["opacities"].append(mop)
            dense["tiles_per_gauss"].append(tiles)
            dense["conics"].append(mcon)
            continue
        rows: dict[str, list[Tensor]] = {k: [] for k in dense}
        for c in range(layout.cameras):
            view = batch_item(batch_item(layout.viewmats, b), c)
            proj = batch_item(batch_item(full, b), c)
            K = batch_item(batch_item(layout.Ks, b), c)
            campos = batch_item(batch_item(centers, b), c) if with_centers else None
            values = layout.colors.at(b, c)
            out = ProjectView.apply(bm, bq, bs, bo,
                                    values if sh_degree is not None else None, view, proj,
                                    campos, K, config, sh_degree, grad_enabled)
            ctr, con, col, radii, tiles, depths, m2d, mop, mcon = out
            colors = col if sh_degree is not None else values
            extras = None if layout.extras is None else layout.extras.at(b, c)
            bg = None if layout.backgrounds is None else batch_item(batch_item(layout.backgrounds, b), c)
            frames.append((b, c, ctr, con, colors, extras, bg,
                           stages.ProjectedGaussians(ctr, con, radii, tiles, depths)))
            rows["radii"].append(radii[:, None].expand(-1, 2))
            rows["means2d"].append(m2d)
            rows["opacities"].append(mop)
            rows["tiles_per_gauss"].append(tiles)
            rows["conics"].append(mcon)
        for name, r in rows.items():
            dense[name].append(r[0][None] if len(r) == 1 else torch.stack(r))
    geometry = {
        name: (per_batch[0] if len(per_batch) == 1 else torch.stack(per_batch)).reshape(
            (layout.batch_count, layout.cameras, layout.n) + tuple(per_batch[0].shape[2:]))
        for name, per_batch in dense.items()
    }
    channels = layout.colors.channels
    # Work that does not need the pair counts is queued before the host
    # read, so the GPU is not left idle while the host prepares it after.
    backgrounds = []
    for (b, c, ctr, con, colors, extras, bg, _state) in frames:
        total = channels + (0 if extras is None else extras.shape[-1]) + 1
        if bg is None:
            packed_bg = _zero_background(ctr.device, total)
        else:
            packed_bg = ctr.new_zeros(total)
            packed_bg[:channels] = bg
        backgrounds.append(packed_bg)
    if not packed:
        training = prepare_training_metadata(geometry, layout, packed=False, absgrad=absgrad)
    # Binning reads the pair counts (and camera status) in one host
    # synchronisation; the packed metadata's visible counts ride along.
    visible = [(f[7].radii > 0).sum() for f in frames] if packed else []
    bins, visible_counts = stages.bin_and_sort_many([f[7] for f in frames], width, height,
                                                    camera_status, tile_mode=tile_mode,
                                                    host_reads=visible)
    if packed:
        training = prepare_training_metadata(geometry, layout, packed=True, absgrad=absgrad,
                                             visible_counts=visible_counts)
    meta = training.values
    meta.update(width=width, height=height, tile_size=16, tile_width=(width + 15) // 16,
                tile_height=(height + 15) // 16, n_cameras=layout.cameras, packed=packed,
                backend="gs3d-b200", with_eval3d=False, supports_means2d_grad=True,
                screen_gradient_mode="projected_mean", tile_mode=tile_mode)
    prepared_stats, statistics_outputs = (
        prepare_statistics(statistics, batch_dims=layout.batch_dims,
                           batch_count=layout.batch_count, cameras=layout.cameras, n=layout.n,
                           width=width, height=height, device=layout.device)
        if statistics else ([], {}))
    blended, alphas = [], []
    for i, (b, c, ctr, con, colors, extras, bg, _state) in enumerate(frames):
        screen = None if training.screen is None else batch_item(batch_item(training.screen, b), c)
        main, alpha = RenderView.apply(ctr, con, colors, extras, screen, backgrounds[i],
                                       bins[i]["ranges"], bins[i]["point_list"],
                                       bins[i]["tile_order"], config,
                                       training.absolute_targets[i],
                                       training.screen_targets[i],
                                       prepared_stats[i] if statistics else None, grad_enabled)
        blended.append(main)
        alphas.append(alpha)
    shape = layout.batch_dims + (layout.cameras, height, width)

    def assemble(parts: list[Tensor]) -> Tensor:
        whole = parts[0] if len(parts) == 1 else torch.stack(parts)
        return whole.reshape(shape + (parts[0].shape[-1],))

    main, alpha = assemble(blended), assemble(alphas)
    features = main
    if layout.extras is not None:
        meta["render_extra_signals"] = main[..., channels:]
        features = main[..., :channels]
    return RasterizationResult(features, alpha, meta, statistics_outputs)
