"""gsplat-signature adapter for AAA-Gaussians (aaa/gsplat.py:17-223).

`rasterization` takes gsplat's arguments and calls aaa.rasterize.  Options
the AAA pipeline cannot honour raise NotImplementedError and malformed
values raise ValueError, under the same conditions as the reference adapter:
eval_3D is always on, eps2d is fixed at 0.3, tiles are 16 pixels, only RGB
/ feature rendering with pinhole cameras and a global shutter.
rasterize_mode selects the EWA opacity compensation ("antialiased") unless
explicit aaa_settings are given.
"""

from __future__ import annotations

import math
from numbers import Integral
from typing import Any, Sequence

from torch import Tensor

from ..statistics import StatisticsRequest
from .api import rasterize
from .config import default_settings
from .settings import ExtendedSettings

# flags and values the AAA pipeline has no counterpart for
_FLAGS = ("sparse_grad", "distributed", "segmented", "with_ut")
_VALUES = ("covars", "radial_coeffs", "tangential_coeffs", "thin_prism_coeffs", "ftheta_coeffs",
           "viewmats_rs", "extra_signals_sh_degree")


def _positive_ints(*values) -> bool:
    return all(not isinstance(v, bool) and isinstance(v, Integral) and v > 0 for v in values)


def _check(options: dict) -> None:
    for name in _FLAGS:
        if options[name]:
            raise NotImplementedError(f"aaa.gsplat.rasterization: {name}=True is not available")
    for name in _VALUES:
        if options[name] is not None:
            raise NotImplementedError(f"aaa.gsplat.rasterization: {name} is not available")
    shutter = getattr(options["rolling_shutter"], "name", options["rolling_shutter"])
    rules = [
        (shutter not in (None, 0, "GLOBAL", "global"), NotImplementedError,
         "a global shutter is required"),
        (options["camera_model"] != "pinhole", NotImplementedError,
         "pinhole cameras are required"),
        (options["with_eval3d"] is False, NotImplementedError,
         "AAA always evaluates Gaussians in 3D (with_eval3d must be None or True)"),
        (options["eps2d"] != 0.3, NotImplementedError,
         "eps2d is fixed at 0.3 by AAA's adaptive filter"),
        (options["tile_size"] not in (None, 16), NotImplementedError,
         "the HIER queues need tile_size=16"),
        (options["render_mode"] != "RGB", NotImplementedError,
         "render_mode must be 'RGB' (colours or arbitrary features); no depth modes"),
        (options["rasterize_mode"] not in ("classic", "antialiased"), ValueError,
         "rasterize_mode must be 'classic' or 'antialiased'"),
        (not _positive_ints(options["width"], options["height"], options["channel_chunk"]),
         ValueError, "width, height and channel_chunk must be positive integers"),
    ]
    near, far, clip = options["near_plane"], options["far_plane"], options["radius_clip"]
    rules += [
        (not math.isfinite(near) or near <= 0 or math.isnan(far) or far <= near, ValueError,
         "need 0 < near_plane < far_plane"),
        (not math.isfinite(clip) or clip < 0, ValueError,
         "radius_clip must be finite and >= 0"),
    ]
    degree = options["sh_degree"]
    rules.append((degree is not None and (isinstance(degree, bool)
                                          or not isinstance(degree, Integral)
                                          or degree not in range(4)),
                  ValueError, "sh_degree must be None or an integer in [0, 3]"))
    for failed, error, message in rules:
        if failed:
            raise error(message)


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
                  aaa_settings: ExtendedSettings | None = None, filter3D: Tensor | None = None,
                  statistics: Sequence[StatisticsRequest] = ()
                  ) -> tuple[Tensor, Tensor, dict[str, Any]]:
    """(render_colors (...,C,H,W,D), render_alphas (...,C,H,W,1), meta) in
    gsplat's layouts; alpha is blended as a constant-one feature."""
    _check(dict(locals()))
    result = rasterize(
        means, quats, scales, opacities, viewmats, Ks, width, height,
        features=colors if sh_degree is None else None,
        sh_coeffs=colors if sh_degree is not None else None, sh_degree=sh_degree,
        backgrounds=backgrounds, extra_features=extra_signals, filter3d=filter3D,
        near_plane=near_plane, far_plane=far_plane, radius_clip=radius_clip, packed=packed,
        absgrad=absgrad,
        settings=(default_settings(antialiased=rasterize_mode == "antialiased")
                  if aaa_settings is None else aaa_settings),
        statistics=statistics)
    if statistics:
        result.meta["statistics"] = result.statistics
    return result.features, result.alpha, result.meta


__all__ = ["rasterization"]
