"""Autograd bridges for one gs3d view (gs3d/autograd.py:1-174).

The reference keeps one Function per view around binning + blending and
separate Functions for projection and SH.  Here projection and SH are one
Function (one forward kernel, one fused backward kernel) and binning +
blending another; gradients reach the same inputs with the same meaning:
means2d receives dL/dcenters and its absgrad the per-pixel |dL/dcenters|
sums (gs3d/autograd.py:386-401).
"""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor
from torch.autograd.function import once_differentiable

from .. import stages
from .._native import check, lib, ptr, stream
from ..camera_prep import ViewConfig
from ..training import AbsGradientTarget


class ProjectView(torch.autograd.Function):
    """Projection + masked SH + metadata for one view (gs3d/api.py:145-189).

    quats_raw is the caller's quaternion tensor and quats its F.normalize
    (computed by the caller without autograd, inputs.py:252); the backward
    kernel applies the normalisation's VJP, so the gradient reaches
    quats_raw without Torch's elementwise backward kernels."""

    @staticmethod
    def forward(ctx: Any, means: Tensor, quats_raw: Tensor, quats: Tensor, scales: Tensor,
                opacities: Tensor, sh: Tensor | None, view: Tensor, full: Tensor,
                campos: Tensor | None, intrinsics: Tensor, config: ViewConfig, sh_degree: int,
                grad_enabled: bool):
        means, quats, scales = means.contiguous(), quats.contiguous(), scales.contiguous()
        quats_raw = quats_raw.contiguous()
        out = stages.project_fused(
            means, quats, scales, opacities.contiguous(), view.contiguous(), full.contiguous(),
            intrinsics.contiguous(), config.width, config.height, config.near, config.far,
            config.radius_clip, sh=None if sh is None else sh.contiguous(),
            sh_degree=sh_degree or 0, campos=None if campos is None else campos.contiguous(),
            need_active=grad_enabled)
        st = out.state
        colors = out.colors if out.colors is not None else means.new_empty((0, 3))
        if grad_enabled and any(ctx.needs_input_grad[:9]):
            ctx.save_for_backward(means, quats, quats_raw, scales, view, full, intrinsics,
                                  st.radii, None if sh is None else sh.contiguous(),
                                  None if campos is None else campos.contiguous(), out.active)
            ctx.config, ctx.sh_degree = config, sh_degree or 0
        ctx.mark_non_differentiable(st.radii, st.tile_counts, st.depths, out.means2d,
                                    out.opacities, out.conics3)
        if sh is None:
            ctx.mark_non_differentiable(colors)
        ctx.set_materialize_grads(False)
        return (st.centers, st.conics, colors, st.radii, st.tile_counts, st.depths, out.means2d,
                out.opacities, out.conics3)

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, g_centers, g_conics, g_colors, *unused):
        if g_centers is None and g_conics is None and g_colors is None:
            return (None,) * 13
        (means, quats, quats_raw, scales, view, full, intrinsics, radii, sh, campos,
         active) = ctx.saved_tensors
        # inputs: 0 means, 1 quats_raw, 2 quats (no grad), 3 scales, 4 opacities,
        # 5 sh, 6 view, 7 full, 8 campos
        needs = ctx.needs_input_grad
        n = len(means)
        cfg = ctx.config
        g_centers = torch.zeros((n, 2), device=means.device) if g_centers is None else g_centers.contiguous()
        g_conics = torch.zeros((n, 4), device=means.device) if g_conics is None else g_conics.contiguous()
        gm = torch.empty_like(means) if needs[0] else None
        gq = torch.empty_like(quats) if needs[1] else None
        gs = torch.empty_like(scales) if needs[3] else None
        go = means.new_empty(n) if needs[4] else None
        gsh = None
        if sh is not None and (needs[5] or (needs[0] and ctx.sh_degree > 0) or needs[8]):
            gsh = torch.empty_like(sh)
        want_cam = needs[6] or needs[7] or needs[8]
        cam = means.new_zeros(35) if want_cam else None
        if gsh is not None:
            gcol = (torch.zeros((n, 3), device=means.device) if g_colors is None
                    else g_colors.contiguous())
        else:
            gcol = None
        if n:
            pin = stages.Args()
            check(lib.splat_project_backward_fused(
                n, pin(means), pin(quats), pin(quats_raw), pin(scales), pin(view), pin(full),
                pin(intrinsics), cfg.width, cfg.height, pin(radii), pin(g_centers),
                pin(g_conics), ptr(gm), ptr(gq), ptr(gs), ptr(go), 0, ptr(cam), ctx.sh_degree,
                0 if sh is None else sh.shape[1], pin(sh), pin(campos), pin(active), pin(gcol), 3,
                ptr(gsh), stream(means.device)), "project_backward_fused")
        gview = cam[:16].reshape(4, 4) if needs[6] else None
        gfull = cam[16:32].reshape(4, 4) if needs[7] else None
        gcampos = cam[32:35].clone() if needs[8] else None
        return (gm, gq, None, gs, go, gsh if needs[5] else None, gview, gfull, gcampos, None,
                None, None, None)


class RenderView(torch.autograd.Function):
    """Blending of one view over pre-binned tiles (gs3d/autograd.py:19-171)."""

    @staticmethod
    def forward(ctx: Any, centers: Tensor, conics: Tensor, colors: Tensor, extras: Tensor | None,
                screen: Tensor | None, background: Tensor, ranges: Tensor, ids: Tensor,
                config: ViewConfig, absolute: AbsGradientTarget | None, statistics,
                grad_enabled: bool) -> Tensor:
        state = stages.ProjectedFootprint(centers, conics)
        bins = dict(ranges=ranges, point_list=ids)
        out = stages.render(state, bins, colors, extras, True, background, config.width,
                            config.height, statistics=statistics)
        if grad_enabled and any(ctx.needs_input_grad[:5]):
            ctx.save_for_backward(centers, conics, colors, extras, background, ranges, ids,
                                  out.transmittance, out.contributors)
            ctx.config, ctx.absolute = config, absolute
        ctx.set_materialize_grads(False)
        return out.features

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, gradient: Tensor | None):
        if gradient is None:
            return (None,) * 12
        centers, conics, colors, extras, background, ranges, ids, final_t, contrib = ctx.saved_tensors
        cfg = ctx.config
        needs = ctx.needs_input_grad
        gc, gq, ga, gb, absolute = stages.render_backward(
            stages.ProjectedFootprint(centers, conics), dict(ranges=ranges, point_list=ids),
            colors, extras, True, background, final_t, contrib, gradient, cfg.width, cfg.height,
            absgrad=ctx.absolute is not None, constant_tail=1, need_a=needs[2],
            need_b=extras is not None and needs[3])
        if ctx.absolute is not None:
            ctx.absolute.write(absolute)
        return (gc if needs[0] else None, gq if needs[1] else None, ga, gb,
                gc if needs[4] else None, None, None, None, None, None, None, None)
