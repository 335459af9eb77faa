"""RaDe-GS autograd bridges (rade/autograd.py:17-189, rade/ops.py:70-242).

The reference wraps binning, rendering, the render backward and the
projection backward into one Function per view, with the projection done
beforehand under no_grad.  Here the projection and the blend are two
Functions joined by ordinary autograd edges (centers, conics, ray planes,
normals): the same gradients, with the SH colours (a separate autograd
Function in both) in between.  The blend Function takes the view's bins
and the training-metadata targets (|d means2d| sums, the means2d leaf).
"""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor
from torch.autograd.function import once_differentiable

from ..training import AbsGradientTarget, ScreenGradientTarget
from . import projection, render
from .projection import ProjectedGaussians, ViewConfig


class Project(torch.autograd.Function):
    """rade/ops.py:70-165 _Project, fused with the SH colours
    (rade/api.py:153-165) and the dense metadata of the same launch:
    differentiable centers, conics, colors, ray planes and normals; radii,
    tile counts, sort distances and the metadata are discrete.  quats_raw
    is normalised in-kernel with Torch's CUDA F.normalize bits and the
    backward applies the normalisation's VJP."""

    @staticmethod
    def forward(ctx: Any, means: Tensor, quats_raw: Tensor, scales: Tensor, opacities: Tensor,
                sh: Tensor | None, view: Tensor, full: Tensor, campos: Tensor | None,
                intrinsics: Tensor, config: ViewConfig, sh_degree: int, grad_enabled: bool):
        means, quats_raw, scales = means.contiguous(), quats_raw.contiguous(), scales.contiguous()
        opacities, view, full = opacities.contiguous(), view.contiguous(), full.contiguous()
        intrinsics = intrinsics.contiguous()
        sh = None if sh is None else sh.contiguous()
        campos = None if campos is None else campos.contiguous()
        out = projection.prepare_fused(means, quats_raw, scales, opacities, view, full,
                                       intrinsics, config, normalize_quats=True, sh=sh,
                                       sh_degree=sh_degree or 0, campos=campos,
                                       need_active=grad_enabled, metadata=True)
        st = out.state
        colors = out.colors if out.colors is not None else means.new_empty((0, 3))
        if grad_enabled and any(ctx.needs_input_grad[:8]):
            ctx.save_for_backward(means, quats_raw, scales, opacities, view, full, intrinsics,
                                  st.radii, sh, campos, out.active)
            ctx.config, ctx.sh_degree = config, sh_degree or 0
        ctx.mark_non_differentiable(st.radii, st.tile_counts, st.depths, out.means2d,
                                    out.opacities, out.conics3)
        if sh is None:
            ctx.mark_non_differentiable(colors)
        ctx.set_materialize_grads(False)
        return (st.centers, st.conics, colors, st.radii, st.tile_counts, st.depths,
                st.ray_planes, st.normals, out.means2d, out.opacities, out.conics3)

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, g_centers, g_conics, g_colors, _radii, _tiles, _depths, g_planes,
                 g_normals, *unused):
        if all(g is None for g in (g_centers, g_conics, g_colors, g_planes, g_normals)):
            return (None,) * 12
        (means, quats_raw, scales, opacities, view, full, intrinsics, radii, sh, campos,
         active) = ctx.saved_tensors
        needs = ctx.needs_input_grad
        # inputs: 0 means, 1 quats_raw, 2 scales, 3 opacities, 4 sh, 5 view, 6 full, 7 campos
        state = ProjectedGaussians(None, None, radii, None, None, None, None)
        gm, gq, gs, go, gv, gp, gsh, gc = projection.backward(
            means, quats_raw, scales, opacities, view, full, intrinsics, ctx.config, state,
            g_centers, g_conics, g_planes, g_normals,
            (needs[0], needs[1], needs[2], needs[3], needs[5], needs[6]),
            normalize_quats=True, sh=sh, sh_degree=ctx.sh_degree, campos=campos, active=active,
            grad_colors=None if g_colors is None else g_colors.contiguous(),
            need_sh=sh is not None and needs[4], need_campos=campos is not None and needs[7])
        return (gm, gq, gs, go, gsh, gv, gp, gc, None, None, None, None)


class Render(torch.autograd.Function):
    """rade/autograd.py:17-189 (binning excluded: the bins come in) and
    rade/ops.py:168-242 _Pixels: the five channel-last images of one view."""

    @staticmethod
    def forward(ctx: Any, centers: Tensor, conics: Tensor, planes: Tensor, normals: Tensor,
                colors: Tensor, extras: Tensor | None, screen: Tensor | None,
                background: Tensor, bins: dict, intrinsics: Tensor, config: ViewConfig,
                absolute: AbsGradientTarget | None, screen_target: ScreenGradientTarget | None,
                statistics, grad_enabled: bool):
        state = ProjectedGaussians(centers, conics, None, None, None, planes, normals)
        out = render.render(state, bins, colors, extras, background, intrinsics, config.width,
                            config.height, statistics)
        if grad_enabled and any(ctx.needs_input_grad[:7]):
            ctx.save_for_backward(centers, conics, planes, normals, colors, extras, background,
                                  intrinsics, out.alpha, out.normals, out.auxiliary,
                                  out.contributors)
            ctx.bins = {k: bins[k] for k in ("ranges", "point_list", "tile_order") if k in bins}
            ctx.config, ctx.absolute, ctx.screen_target = config, absolute, screen_target
        ctx.set_materialize_grads(False)
        # colour and extra channels as two outputs (views of the blended
        # buffer): the backward kernel reads their upstream gradients from two
        # images, where slicing one output would make autograd scatter each
        # into a zero-filled buffer of all channels
        split = colors.shape[1]
        ctx.split = split
        if extras is None:
            empty = out.features.new_empty(out.features.shape[:-1] + (0,))
            ctx.mark_non_differentiable(empty)
            feats, extra_image = out.features, empty
        else:
            feats, extra_image = out.features[..., :split], out.features[..., split:]
        return feats, extra_image, out.alpha, out.depth, out.median, out.normals

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, g_colors, g_extras, *geometry: Tensor | None):
        if all(g is None for g in (g_colors, g_extras) + geometry):
            return (None,) * 15
        (centers, conics, planes, normals, colors, extras, background, intrinsics, alpha,
         normal_image, aux, contrib) = ctx.saved_tensors
        cfg = ctx.config
        needs = ctx.needs_input_grad
        direct = ctx.absolute.direct_buffer() if ctx.absolute is not None else None
        screen_direct = (ctx.screen_target.direct_buffer()
                         if needs[6] and ctx.screen_target is not None else None)
        state = ProjectedGaussians(centers, conics, None, None, None, planes, normals)
        # the colour and extra upstreams are read in place (None: zero)
        gradients = ((g_colors, g_extras if extras is not None else None),) + tuple(geometry)
        gc, gq, ga, gb, gp, gn, absolute = render.backward(
            state, ctx.bins, colors, extras, background, intrinsics,
            render.RenderedPixels(None, alpha, None, None, normal_image, aux, contrib),
            gradients, cfg.width, cfg.height,
            absgrad=ctx.absolute is not None, need_colors=needs[4],
            need_extras=extras is not None and needs[5], centers_out=screen_direct,
            absolute_out=direct)
        if ctx.absolute is not None and direct is None:
            ctx.absolute.write(absolute)
        g_screen = None
        if needs[6]:
            if ctx.screen_target is not None:
                if screen_direct is None:
                    ctx.screen_target.add(gc)
            else:
                g_screen = gc
        return (gc if needs[0] else None, gq if needs[1] else None, gp if needs[2] else None,
                gn if needs[3] else None, ga, gb, g_screen, None, None, None, None, None, None,
                None, None)
