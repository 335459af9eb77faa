"""gsplat-signature adapter for original 3DGS (gs3d/gsplat.py:1-197).

Translates gsplat's `rasterization` arguments to gs3d.rasterize and rejects
what gs3d does not support, with the reference's exception types and
messages.  means2d stays in CUDA raster coordinates; the adapter keeps
gsplat's near_plane=0.01 default.
"""

from __future__ import annotations

import math
from numbers import Integral
from typing import Any, Sequence

from torch import Tensor

from ..statistics import StatisticsRequest
from .api import rasterize


def _validate_options(width, height, near_plane, far_plane, radius_clip, eps2d, sh_degree,
                      tile_size, render_mode, rasterize_mode, channel_chunk, camera_model,
                      with_eval3d, rolling_shutter, unsupported, unsupported_values) -> None:
    for name, enabled in unsupported.items():
        if enabled:
            raise NotImplementedError(f"3DGS/B200 gsplat adapter does not support {name}=True")
    for name, value in unsupported_values.items():
        if value is not None:
            raise NotImplementedError(f"3DGS/B200 gsplat adapter does not support {name}")
    shutter = getattr(rolling_shutter, "name", rolling_shutter)
    if shutter not in (None, 0, "GLOBAL", "global"):
        raise NotImplementedError("only global shutter is supported")
    if camera_model != "pinhole":
        raise NotImplementedError("only pinhole cameras are supported")
    if with_eval3d is True:
        raise NotImplementedError(
            "original 3DGS uses projected 2D conics; with_eval3d=True is unsupported")
    if eps2d != 0.3:
        raise NotImplementedError("original 3DGS currently has fixed eps2d=0.3")
    if tile_size not in (None, 16):
        raise NotImplementedError("original 3DGS currently requires tile_size=16")
    if render_mode != "RGB":
        raise NotImplementedError(
            "3DGS/B200 supports render_mode='RGB' for RGB or arbitrary features; "
            "depth rendering is not implemented")
    if rasterize_mode != "classic":
        raise NotImplementedError("original 3DGS supports rasterize_mode='classic' only")
    if any(isinstance(v, bool) or not isinstance(v, Integral) or v <= 0
           for v in (width, height, channel_chunk)):
        raise ValueError("width, height and channel_chunk must be positive integers")
    if (not math.isfinite(near_plane) or near_plane <= 0 or math.isnan(far_plane)
            or far_plane <= near_plane):
        raise ValueError("require 0 < near_plane < far_plane")
    if not math.isfinite(radius_clip) or radius_clip < 0:
        raise ValueError("radius_clip must be finite and nonnegative")
    if sh_degree is not None and (isinstance(sh_degree, bool) or not isinstance(sh_degree, Integral)
                                  or sh_degree not in range(4)):
        raise ValueError("sh_degree must be None or an integer in [0,3]")


def rasterization(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor,
                  colors: Tensor | None, viewmats: Tensor, Ks: Tensor, width: int, height: int,
                  near_plane: float = 0.01, far_plane: float = 10000000000.0,
                  radius_clip: float = 0.0, eps2d: float = 0.3, sh_degree: int | None = None,
                  packed: bool = True, tile_size: int | None = 16,
                  backgrounds: Tensor | None = None, render_mode: str = "RGB",
                  sparse_grad: bool = False, absgrad: bool = False,
                  rasterize_mode: str = "classic", channel_chunk: int = 32,
                  distributed: bool = False, camera_model: str = "pinhole",
                  segmented: bool = False, covars: Tensor | None = None, with_ut: bool = False,
                  with_eval3d: bool | None = None, radial_coeffs: Tensor | None = None,
                  tangential_coeffs: Tensor | None = None,
                  thin_prism_coeffs: Tensor | None = None, ftheta_coeffs: object | None = None,
                  rolling_shutter: object | None = None, viewmats_rs: Tensor | None = None, *,
                  extra_signals: Tensor | None = None,
                  extra_signals_sh_degree: int | None = None,
                  statistics: Sequence[StatisticsRequest] = (),
                  tile_mode: str = "radius") -> tuple[Tensor, Tensor, dict[str, Any]]:
    """Return (features, alpha, meta) from the original-3DGS pipeline."""
    _validate_options(
        width, height, near_plane, far_plane, radius_clip, eps2d, sh_degree, tile_size,
        render_mode, rasterize_mode, channel_chunk, camera_model, with_eval3d, rolling_shutter,
        dict(sparse_grad=sparse_grad, distributed=distributed, segmented=segmented,
             with_ut=with_ut),
        dict(covars=covars, radial_coeffs=radial_coeffs, tangential_coeffs=tangential_coeffs,
             thin_prism_coeffs=thin_prism_coeffs, ftheta_coeffs=ftheta_coeffs,
             viewmats_rs=viewmats_rs, extra_signals_sh_degree=extra_signals_sh_degree))
    result = rasterize(
        means, quats, scales, opacities, viewmats, Ks, width, height,
        features=colors if sh_degree is None else None,
        sh_coeffs=colors if sh_degree is not None else None, sh_degree=sh_degree,
        backgrounds=backgrounds, extra_features=extra_signals, near_plane=near_plane,
        far_plane=far_plane, radius_clip=radius_clip, packed=packed, absgrad=absgrad,
        statistics=statistics, tile_mode=tile_mode)
    if statistics:
        result.meta["statistics"] = result.statistics
    return result.features, result.alpha, result.meta


__all__ = ["rasterization"]
