"""RaDe-GS blend stage (rade/render.py:550-670 render/backward) on the
sm_100a kernels: colour, alpha, expected and median depth and normals in one
traversal, and the reverse replay with warp-reduced atomics."""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from .. import _native as nv
from .. import stages
from .._native import check, lib, ptr
from .projection import ProjectedGaussians


@dataclass(slots=True)
class RenderedPixels:
    """rade/render.py:32-47, with the five images the reference slices out of
    its planar (C+6, H, W) buffer written by the kernel as separate dense
    channel-last tensors: features (H, W, C), alpha, expected depth and
    median depth (H, W, 1), normals (H, W, 3); plus auxiliary (2, H, W)
    (depth times the ray scale, normal length) and contributors (2, H, W)
    (last and median contributor)."""

    features: Tensor
    alpha: Tensor
    depth: Tensor
    median: Tensor
    normals: Tensor
    auxiliary: Tensor
    contributors: Tensor

    def images(self) -> tuple[Tensor, ...]:
        """Feature, alpha, expected depth, median depth and normal HWC images."""
        return self.features, self.alpha, self.depth, self.median, self.normals

    def planar(self) -> Tensor:
        """The reference's (C+6, H, W) layout (a copy)."""
        return torch.cat(self.images(), -1).permute(2, 0, 1)


def _split(colors: Tensor, extras: Tensor | None):
    a = colors.contiguous()
    b = None if extras is None else extras.contiguous()
    return a, b, a.shape[1], (0 if b is None else b.shape[1])


def render(state: ProjectedGaussians, bins: dict, colors: Tensor, extras: Tensor | None,
           background: Tensor, intrinsics: Tensor, width: int, height: int,
           statistics=None) -> RenderedPixels:
    """rade/render.py:550-601.  Channels: colors then extras; background
    covers all of them."""
    pin = stages.Args()
    a, b, ca, cb = _split(colors, extras)
    dev = a.device
    channels = ca + cb
    out = RenderedPixels(a.new_empty((height, width, channels)), a.new_empty((height, width, 1)),
                         a.new_empty((height, width, 1)), a.new_empty((height, width, 1)),
                         a.new_empty((height, width, 3)), a.new_empty((2, height, width)),
                         torch.empty((2, height, width), dtype=torch.int32, device=dev))
    if statistics is None:
        stat = (0, 0, None, None, None)
    else:
        mask = sum(1 << r for r, kind in enumerate(statistics.key) if kind == 1)
        stat = (len(statistics.key), mask, ptr(statistics.pixel_values),
                ptr(statistics.counts), ptr(statistics.sums))
    with stages._timed("rade_render_forward", dev):
        check(lib.splat_rade_render_forward(
            width, height, ptr(bins["ranges"]), ptr(bins["point_list"]), len(bins["point_list"]),
            len(state.centers), pin(state.centers), pin(state.conics), pin(state.ray_planes),
            pin(state.normals), ptr(a), ca, ca, ptr(b), cb, cb, pin(background),
            pin(intrinsics), ptr(out.features), channels, 1, ptr(out.alpha), 1, ptr(out.depth), 1,
            ptr(out.median), 1, ptr(out.normals), 3, 1, ptr(out.auxiliary),
            ptr(out.contributors), *stat, ptr(stages.tile_order(bins)), nv.stream(dev)),
            "rade_render_forward")
    return out


def _upstream(g: Tensor | None, channels: int):
    """(pointer source, pixel stride, channel stride) of an (H, W, k) image gradient."""
    if g is None:
        return None, 0, 0
    g = g.contiguous()
    return g, channels, 1


def backward(state: ProjectedGaussians, bins: dict, colors: Tensor, extras: Tensor | None,
             background: Tensor, intrinsics: Tensor, output: RenderedPixels,
             gradients: tuple[Tensor | None, ...], width: int, height: int, *,
             absgrad: bool = False, need_colors: bool = True, need_extras: bool = True,
             centers_out: Tensor | None = None, absolute_out: Tensor | None = None):
    """rade/render.py:604-670.  gradients: upstream of (features, alpha,
    depth, median depth, normals), each (H, W, k) or None; the features'
    upstream is one (H, W, C) image or a pair (colours (H, W, ch_a) or None,
    extras (H, W, ch_b) or None), read in place.  Returns grads of
    (centers, conics, colors, extras, ray_planes, normals, |centers|)."""
    pin = stages.Args()
    a, b, ca, cb = _split(colors, extras)
    channels = ca + cb
    g0 = gradients[0]
    if isinstance(g0, tuple):
        gf, pf, cf = _upstream(g0[0], ca)
        ge, pe, ce = _upstream(g0[1], cb)
        up_c, up_e = pin(gf), pin(ge)
    else:
        # one image: the extra channels start ca floats into each pixel
        gf, pf, cf = _upstream(g0, channels)
        pe, ce = pf, cf
        up_c = pin(gf)
        up_e = None if up_c is None or cb == 0 else up_c + 4 * ca
    ga, pa, _ = _upstream(gradients[1], 1)
    gd, pd, _ = _upstream(gradients[2], 1)
    gm, pm, _ = _upstream(gradients[3], 1)
    gn, pn, cn = _upstream(gradients[4], 3)
    centers = centers_out if centers_out is not None else torch.zeros_like(state.centers)
    conics = torch.zeros_like(state.conics)
    g_colors = torch.zeros_like(a) if need_colors else None
    g_extras = torch.zeros_like(b) if (b is not None and need_extras) else None
    planes = torch.zeros_like(state.ray_planes)
    normals = torch.zeros_like(state.normals)
    if absgrad:
        absolute = absolute_out if absolute_out is not None else torch.zeros_like(state.centers)
    else:
        absolute = None
    with stages._timed("rade_render_backward", a.device):
        check(lib.splat_rade_render_backward(
            width, height, ptr(bins["ranges"]), ptr(bins["point_list"]), len(bins["point_list"]),
            len(state.centers), pin(state.centers), pin(state.conics), pin(state.ray_planes),
            pin(state.normals), ptr(a), ca, ca, ptr(b), cb, cb, pin(background),
            pin(intrinsics), pin(output.alpha), 1, pin(output.normals), 3, 1,
            pin(output.auxiliary), pin(output.contributors), up_c, pf, cf, up_e, pe, ce, pin(ga), pa,
            pin(gd), pd, pin(gm), pm,
            pin(gn), pn, cn, ptr(centers), ptr(conics), ptr(g_colors), ptr(g_extras),
            ptr(absolute), ptr(planes), ptr(normals), ptr(stages.tile_order(bins)),
            nv.stream(a.device)), "rade_render_backward")
    return centers, conics, g_colors, g_extras, planes, normals, absolute
