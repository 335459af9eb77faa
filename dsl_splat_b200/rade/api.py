"""RaDe-GS entry point (rade/api.py:1-275) on the sm_100a kernels.

Same signature, validation, batching, metadata and result type as the
reference.  Per call: one camera launch for all views; per view one
projection launch (ray planes, normals, radial sort distance) and the SH
colours; binning of all views with a single host read of their pair counts;
one blend launch per view producing colour, alpha, expected and median depth
and normals together.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Sequence

import torch
from torch import Tensor

from .. import stages
from ..camera_prep import prepare_cameras, prepare_cameras_with_centers
from ..cameras import validate_camera_options
from ..gs3d.api import _check_sh
from ..inputs import batch_item, normalize_inputs
from ..statistics import StatisticsRequest, prepare_statistics
from ..training import prepare_training_metadata
from .autograd import Project, Render
from .projection import ProjectedGaussians, ViewConfig


@dataclass(slots=True)
class RasterizationResult:
    """Channel-last views of the rendered images and training metadata
    (rade/api.py:25-47)."""

    features: Tensor
    alpha: Tensor
    depth: Tensor
    median_depth: Tensor
    normals: Tensor
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


def validate_kernel_size(kernel_size) -> None:
    """rade/api.py:82-83."""
    if not math.isfinite(kernel_size) or kernel_size < 0:
        raise ValueError("kernel_size must be finite and nonnegative")


def rasterize(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor, viewmats: Tensor,
              Ks: Tensor, width: int, height: int, *, features: Tensor | None = None,
              sh_coeffs: Tensor | None = None, sh_degree: int | None = None,
              backgrounds: Tensor | None = None, extra_features: Tensor | None = None,
              near_plane: float = 0.2, far_plane: float = math.inf, radius_clip: float = 0.0,
              kernel_size: float = 0.0, packed: bool = False, absgrad: bool = False,
              statistics: Sequence[StatisticsRequest] = ()) -> RasterizationResult:
    """Render RaDe-GS features, alpha, expected/median Z depth and normals.

    Inputs use OpenCV world-to-camera matrices and channel-last images.
    Scales and opacities are activated and quaternions are normalized.  Depth
    is the ray-plane approximation converted to camera Z, the median depth
    the last contributor whose incoming transmittance exceeds 0.5, normals
    unit camera-space vectors (zero where nothing was blended).  kernel_size
    dilates the 2D covariance and compensates opacity.  Intrinsics/background
    gradients are unsupported.
    """
    validate_kernel_size(kernel_size)
    validate_camera_options(width, height, near_plane, far_plane, radius_clip)
    sh_degree = _check_sh(sh_coeffs, sh_degree, features)
    # quaternions reach the projection kernels raw: they apply inputs.py:252's
    # F.normalize with Torch's CUDA bits and its VJP in the backward
    layout = normalize_inputs(means, quats, scales, opacities,
                              features if sh_coeffs is None else sh_coeffs, viewmats, Ks,
                              backgrounds, extra_features, None, sh_degree,
                              normalize_quats=False)
    with_centers = sh_degree is not None and sh_degree > 0
    camera_status: list = []
    if with_centers:
        full, centers = prepare_cameras_with_centers(layout.viewmats, layout.Ks, width, height,
                                                     camera_status)
    else:
        full = prepare_cameras(layout.viewmats, layout.Ks, width, height, camera_status)
        centers = None
    config = ViewConfig(width, height, near_plane, far_plane, radius_clip, "radius",
                        float(kernel_size))
    grad_enabled = torch.is_grad_enabled()
    frames = []
    dense: dict[str, list[Tensor]] = {k: [] for k in ("radii", "means2d", "opacities",
                                                      "tiles_per_gauss", "conics")}
    for b in range(layout.batch_count):
        bm, bq = layout.means[b], layout.quats[b]
        bs, bo = layout.scales[b], layout.opacities[b]
        rows: dict[str, list[Tensor]] = {k: [] for k in dense}
        for c in range(layout.cameras):
            view = batch_item(batch_item(layout.viewmats, b), c)
            proj = batch_item(batch_item(full, b), c)
            K = batch_item(batch_item(layout.Ks, b), c).contiguous()
            values = layout.colors.at(b, c)
            campos = batch_item(batch_item(centers, b), c) if with_centers else None
            # one launch: projection, SH colours on means - campos, metadata
            (ctr, con, colors, radii, tiles, depths, planes, normals, m2d, mop,
             mcon) = Project.apply(bm, bq, bs, bo, values if sh_degree is not None else None,
                                   view, proj, campos, K, config, sh_degree, grad_enabled)
            state = ProjectedGaussians(ctr, con, radii, tiles, depths, planes, normals)
            if sh_degree is not None:
                values = colors
            extras = None if layout.extras is None else layout.extras.at(b, c)
            bg = (None if layout.backgrounds is None
                  else batch_item(batch_item(layout.backgrounds, b), c))
            frames.append((b, c, state, values, extras, bg, K))
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
    backgrounds_packed = []
    for (_b, _c, state, values, extras, bg, _K) in frames:
        total = channels + (0 if extras is None else extras.shape[-1])
        packed_bg = state.centers.new_zeros(total)
        if bg is not None:
            packed_bg[:channels] = bg
        backgrounds_packed.append(packed_bg)
    if not packed:
        training = prepare_training_metadata(geometry, layout, packed=False, absgrad=absgrad)
    visible = [(f[2].radii > 0).sum() for f in frames] if packed else []
    bins, visible_counts = stages.bin_and_sort_many([f[2] for f in frames], width, height,
                                                    camera_status, host_reads=visible)
    if packed:
        training = prepare_training_metadata(geometry, layout, packed=True, absgrad=absgrad,
                                             visible_counts=visible_counts)
    meta = training.values
    meta.update(width=width, height=height, tile_size=16, tile_width=(width + 15) // 16,
                tile_height=(height + 15) // 16, n_cameras=layout.cameras, packed=packed,
                backend="rade-b200", with_eval3d=False, supports_means2d_grad=True,
                screen_gradient_mode="projected_mean")
    prepared_stats, statistics_outputs = (
        prepare_statistics(statistics, batch_dims=layout.batch_dims,
                           batch_count=layout.batch_count, cameras=layout.cameras, n=layout.n,
                           width=width, height=height, device=layout.device)
        if statistics else ([], {}))
    images = []
    for i, (b, c, state, values, extras, _bg, K) in enumerate(frames):
        screen = None if training.screen is None else batch_item(batch_item(training.screen, b), c)
        images.append(Render.apply(
            state.centers, state.conics, state.ray_planes, state.normals, values, extras, screen,
            backgrounds_packed[i], bins[i], K, config, training.absolute_targets[i],
            training.screen_targets[i], prepared_stats[i] if statistics else None, grad_enabled))
    shape = layout.batch_dims + (layout.cameras, height, width)

    def assemble(values: tuple[Tensor, ...]) -> Tensor:
        # each output keeps its own autograd edge (rade/api.py:253-260); one
        # view needs no stacking copy: the blend wrote a dense tensor per output
        whole = values[0].unsqueeze(0) if len(values) == 1 else torch.stack(values)
        return whole.reshape(shape + (values[0].shape[-1],))

    main_features, extra_image, alpha, depth, median, normals = (
        assemble(v) for v in zip(*images))
    if layout.extras is not None:
        meta["render_extra_signals"] = extra_image
    meta.update(depth=depth, median_depth=median, normals=normals)
    return RasterizationResult(main_features, alpha, depth, median, normals, meta,
                               statistics_outputs)
