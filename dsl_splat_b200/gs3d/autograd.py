"""Autograd bridges for one gs3d view (gs3d/autograd.py:1-174).

The reference keeps one Function per view around binning + blending and
separate Functions for projection and SH.  Here projection and SH are one
Function (one forward kernel, one fused backward kernel) and binning +
blending another; gradients reach the same inputs with the same meaning:
means2d receives dL/dcenters and its absgrad the per-pixel |dL/dcenters|
sums (gs3d/autograd.py:120-140).
"""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor
from torch.autograd.function import once_differentiable

from .. import sharding, stages
from .._native import check, lib, ptr, stream
from ..camera_prep import ViewConfig
from ..training import AbsGradientTarget, ScreenGradientTarget


class ProjectView(torch.autograd.Function):
    """Projection + masked SH + metadata for one view (gs3d/api.py:145-189).

    quats_raw is the caller's quaternion tensor: the kernels normalise it
    with the bits of Torch's CUDA F.normalize (inputs.py:252) and the
    backward applies the normalisation's VJP, so the gradient reaches
    quats_raw without Torch's normalize kernels or their backward."""

    @staticmethod
    def forward(ctx: Any, means: Tensor, quats_raw: Tensor, scales: Tensor, opacities: Tensor,
                sh: Tensor | None, view: Tensor, full: Tensor, campos: Tensor | None,
                intrinsics: Tensor, config: ViewConfig, sh_degree: int, grad_enabled: bool):
        means, quats_raw, scales = means.contiguous(), quats_raw.contiguous(), scales.contiguous()
        out = stages.project_fused(
            means, quats_raw, scales, opacities.contiguous(), view.contiguous(),
            full.contiguous(), intrinsics.contiguous(), config.width, config.height, config.near,
            config.far, config.radius_clip, sh=None if sh is None else sh.contiguous(),
            sh_degree=sh_degree or 0, campos=None if campos is None else campos.contiguous(),
            need_active=grad_enabled, normalize_quats=True, tile_mode=config.tile_mode)
        st = out.state
        colors = out.colors if out.colors is not None else means.new_empty((0, 3))
        sync = sharding.current_sync() if grad_enabled else None
        if (sync is not None and any(ctx.needs_input_grad[:5])
                and sync.claims(means, quats_raw, scales, opacities, sh)):
            sync.register_view()
        else:
            sync = None
        ctx.sync = sync
        if grad_enabled and any(ctx.needs_input_grad[:8]):
            ctx.save_for_backward(means, quats_raw, scales, view, full, intrinsics, st.radii,
                                  None if sh is None else sh.contiguous(),
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
        # a GradientSync counts every view's backward (the last one reduces),
        # so a view without upstream gradients still runs, on zeros
        if g_centers is None and g_conics is None and g_colors is None and ctx.sync is None:
            return (None,) * 12
        means, quats_raw, scales, view, full, intrinsics, radii, sh, campos, active = ctx.saved_tensors
        # inputs: 0 means, 1 quats_raw, 2 scales, 3 opacities, 4 sh, 5 view, 6 full, 7 campos
        needs = ctx.needs_input_grad
        n = len(means)
        cfg = ctx.config
        sync = ctx.sync
        g_centers = torch.zeros((n, 2), device=means.device) if g_centers is None else g_centers.contiguous()
        g_conics = torch.zeros((n, 4), device=means.device) if g_conics is None else g_conics.contiguous()
        if sync is not None:
            # per-Gaussian gradients accumulate in the sync's buffers
            buffers, accumulate, last = sync.begin_view()
            gm, gq, gs, go = (buffers.get(k) for k in ("means", "quats", "scales", "opacities"))
            gsh = buffers.get("sh")
            if (gsh is None and sh is not None and ctx.sh_degree > 0
                    and (gm is not None or needs[7])):
                gsh = torch.empty_like(sh)  # direction gradient only; values unused
        else:
            accumulate, last = False, False
            gm = torch.empty_like(means) if needs[0] else None
            gq = torch.empty_like(quats_raw) if needs[1] else None
            gs = torch.empty_like(scales) if needs[2] else None
            go = means.new_empty(n) if needs[3] else None
            gsh = None
            if sh is not None and (needs[4] or (needs[0] and ctx.sh_degree > 0) or needs[7]):
                gsh = torch.empty_like(sh)
        want_cam = needs[5] or needs[6] or needs[7]
        cam = means.new_zeros(35) if want_cam else None
        if gsh is not None:
            gcol = (torch.zeros((n, 3), device=means.device) if g_colors is None
                    else g_colors.contiguous())
        else:
            gcol = None

        def launch(lo: int, hi: int) -> None:
            def rows(t):
                return None if t is None else t[lo:hi]
            pin = stages.Args()
            check(lib.splat_project_backward_fused(
                hi - lo, pin(rows(means)), None, pin(rows(quats_raw)), pin(rows(scales)),
                pin(view), pin(full), pin(intrinsics), cfg.width, cfg.height, pin(rows(radii)),
                pin(rows(g_centers)), pin(rows(g_conics)), ptr(rows(gm)), ptr(rows(gq)),
                ptr(rows(gs)), ptr(rows(go)), int(accumulate), ptr(cam), ctx.sh_degree,
                0 if sh is None else sh.shape[1], pin(rows(sh)), pin(campos), pin(rows(active)),
                pin(rows(gcol)), 3, ptr(rows(gsh)), stream(means.device)),
                "project_backward_fused")

        if n and sync is not None and last:
            # bucket b's all-reduce is queued right behind its kernel, so it
            # runs on NCCL's stream while bucket b+1 computes
            for lo, hi in sharding.bucket_bounds(n, sync.buckets):
                launch(lo, hi)
                sync.reduce_range(lo, hi)
        elif n:
            launch(0, n)
        if sync is not None:
            if last:
                sync.finish()
            gm = gq = gs = go = None
            gsh = None
        gview = cam[:16].reshape(4, 4) if needs[5] else None
        gfull = cam[16:32].reshape(4, 4) if needs[6] else None
        gcampos = cam[32:35].clone() if needs[7] else None
        return (gm, gq, gs, go, gsh if needs[4] else None, gview, gfull, gcampos, None, None,
                None, None)


class ProjectViews(torch.autograd.Function):
    """ProjectView for every camera of a batch in one launch each way
    (gs3d/api.py:132-189's per-camera loop fused: splat_project_forward_views
    and splat_project_backward_views).

    Outputs: per camera its centres, conics and colours (separate tensors,
    so each view's gradient arrives on its own and nothing materialises a
    (views, n, ...) gradient), then the stacked (views, n, ...) radii, tile
    counts, depths and dense metadata.  The backward sums the views inside
    the kernel (one read of every Gaussian's inputs, one write of every
    gradient); when pose gradients are requested it runs the per-view kernel
    once per camera instead."""

    @staticmethod
    def forward(ctx: Any, means: Tensor, quats_raw: Tensor, scales: Tensor, opacities: Tensor,
                sh: Tensor | None, views: Tensor, fulls: Tensor, campos: Tensor | None,
                intrinsics: Tensor, config: ViewConfig, sh_degree: int, grad_enabled: bool):
        means, quats_raw, scales = means.contiguous(), quats_raw.contiguous(), scales.contiguous()
        sh = None if sh is None else sh.contiguous()
        views, fulls, intrinsics = views.contiguous(), fulls.contiguous(), intrinsics.contiguous()
        campos = None if campos is None else campos.contiguous()
        out = stages.project_views(
            means, quats_raw, scales, opacities.contiguous(), views, fulls, intrinsics,
            config.width, config.height, config.near, config.far, config.radius_clip, sh=sh,
            sh_degree=sh_degree or 0, campos=campos, need_active=grad_enabled,
            normalize_quats=True, tile_mode=config.tile_mode)
        V = views.shape[0]
        colors = out.colors if out.colors is not None else [means.new_empty((0, 3))] * V
        sync = sharding.current_sync() if grad_enabled else None
        if (sync is not None and any(ctx.needs_input_grad[:5])
                and sync.claims(means, quats_raw, scales, opacities, sh)):
            sync.register_view()
        else:
            sync = None
        ctx.sync = sync
        if grad_enabled and any(ctx.needs_input_grad[:8]):
            ctx.save_for_backward(means, quats_raw, scales, views, fulls, intrinsics, out.radii,
                                  sh, campos, out.active)
            ctx.config, ctx.sh_degree = config, sh_degree or 0
        ctx.mark_non_differentiable(out.radii, out.tile_counts, out.depths, out.means2d,
                                    out.opacities, out.conics3)
        if sh is None:
            ctx.mark_non_differentiable(*colors)
        ctx.set_materialize_grads(False)
        return (*out.centers, *out.conics, *colors, out.radii, out.tile_counts, out.depths,
                out.means2d, out.opacities, out.conics3)

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, *grads):
        means, quats_raw, scales, views, fulls, intrinsics, radii, sh, campos, active = \
            ctx.saved_tensors
        V, n = views.shape[0], len(means)
        g_centers, g_conics, g_colors = grads[:V], grads[V:2 * V], grads[2 * V:3 * V]
        needs = ctx.needs_input_grad
        cfg, sync = ctx.config, ctx.sync
        if sync is None and all(g is None for g in grads[:3 * V]):
            return (None,) * 12
        dev = means.device
        g_centers = [torch.zeros((n, 2), device=dev) if g is None else g.contiguous()
                     for g in g_centers]
        g_conics = [torch.zeros((n, 4), device=dev) if g is None else g.contiguous()
                    for g in g_conics]
        if sync is not None:
            buffers, accumulate, last = sync.begin_view()
            gm, gq, gs, go = (buffers.get(k) for k in ("means", "quats", "scales", "opacities"))
            gsh = buffers.get("sh")
            if (gsh is None and sh is not None and ctx.sh_degree > 0
                    and (gm is not None or needs[7])):
                gsh = torch.empty_like(sh)  # direction gradient only; values unused
        else:
            accumulate, last = False, False
            gm = torch.empty_like(means) if needs[0] else None
            gq = torch.empty_like(quats_raw) if needs[1] else None
            gs = torch.empty_like(scales) if needs[2] else None
            go = means.new_empty(n) if needs[3] else None
            gsh = None
            if sh is not None and (needs[4] or (needs[0] and ctx.sh_degree > 0) or needs[7]):
                gsh = torch.empty_like(sh)
        gcol = None
        if gsh is not None:
            gcol = [torch.zeros((n, 3), device=dev) if g is None else g.contiguous()
                    for g in g_colors]
        want_cam = needs[5] or needs[6] or needs[7]
        cams = means.new_zeros((V, 35)) if want_cam else None
        K = 0 if sh is None else sh.shape[1]

        def launch(lo: int, hi: int) -> None:
            def rows(t):
                return None if t is None else t[lo:hi]
            pin = stages.Args()
            if cams is None:
                check(lib.splat_project_backward_views(
                    V, hi - lo, pin(rows(means)), None, pin(rows(quats_raw)), pin(rows(scales)),
                    pin(views), pin(fulls), pin(intrinsics), cfg.width, cfg.height,
                    stages.pointer_table(r[lo:hi] for r in radii),
                    stages.pointer_table(g[lo:hi] for g in g_centers),
                    stages.pointer_table(g[lo:hi] for g in g_conics), ptr(rows(gm)),
                    ptr(rows(gq)), ptr(rows(gs)), ptr(rows(go)), int(accumulate),
                    ctx.sh_degree, K, pin(rows(sh)), pin(campos),
                    stages.pointer_table(a[lo:hi] for a in active) if gsh is not None else None,
                    stages.pointer_table(g[lo:hi] for g in gcol) if gsh is not None else None, 3,
                    ptr(rows(gsh)), stream(dev)), "project_backward_views")
                return
            # pose gradients: the per-view kernel once per camera (its camera
            # reduction), views after the first accumulating
            for v in range(V):
                check(lib.splat_project_backward_fused(
                    hi - lo, pin(rows(means)), None, pin(rows(quats_raw)), pin(rows(scales)),
                    pin(views[v]), pin(fulls[v]), pin(intrinsics[v]), cfg.width, cfg.height,
                    pin(radii[v, lo:hi]), pin(g_centers[v][lo:hi]), pin(g_conics[v][lo:hi]),
                    ptr(rows(gm)), ptr(rows(gq)), ptr(rows(gs)), ptr(rows(go)),
                    int(accumulate or v > 0), ptr(cams[v]), ctx.sh_degree, K, pin(rows(sh)),
                    pin(None if campos is None else campos[v]),
                    pin(None if active is None or gsh is None else active[v, lo:hi]),
                    pin(None if gcol is None else gcol[v][lo:hi]), 3, ptr(rows(gsh)),
                    stream(dev)), "project_backward_fused")

        if n and sync is not None and last:
            for lo, hi in sharding.bucket_bounds(n, sync.buckets):
                launch(lo, hi)
                sync.reduce_range(lo, hi)
        elif n:
            launch(0, n)
        if sync is not None:
            if last:
                sync.finish()
            gm = gq = gs = go = gsh = None
        gview = cams[:, :16].reshape(V, 4, 4) if needs[5] else None
        gfull = cams[:, 16:32].reshape(V, 4, 4) if needs[6] else None
        gcampos = cams[:, 32:35].clone() if needs[7] else None
        return (gm, gq, gs, go, gsh if needs[4] else None, gview, gfull, gcampos, None, None,
                None, None)


class RenderView(torch.autograd.Function):
    """Blending of one view over pre-binned tiles (gs3d/autograd.py:19-171).

    Returns the blended channels before the constant one (colours, then
    extras) and the alpha channel as two dense buffers, so neither output is
    a slice whose backward would materialise a zero-filled full image."""

    @staticmethod
    def forward(ctx: Any, centers: Tensor, conics: Tensor, colors: Tensor, extras: Tensor | None,
                screen: Tensor | None, background: Tensor, ranges: Tensor, ids: Tensor,
                order: Tensor, config: ViewConfig, absolute: AbsGradientTarget | None,
                screen_target: ScreenGradientTarget | None, statistics, grad_enabled: bool):
        state = stages.ProjectedFootprint(centers, conics)
        bins = dict(ranges=ranges, point_list=ids, tile_order=order)
        out = stages.render(state, bins, colors, extras, True, background, config.width,
                            config.height, statistics=statistics, separate_alpha=True)
        if grad_enabled and any(ctx.needs_input_grad[:5]):
            ctx.save_for_backward(centers, conics, colors, extras, background, ranges, ids,
                                  order, out.transmittance, out.contributors)
            ctx.config, ctx.absolute, ctx.screen_target = config, absolute, screen_target
        ctx.set_materialize_grads(False)
        return out.features, out.alpha

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, g_features: Tensor | None, g_alpha: Tensor | None):
        if g_features is None and g_alpha is None:
            return (None,) * 14
        centers, conics, colors, extras, background, ranges, ids, order, final_t, contrib = \
            ctx.saved_tensors
        cfg = ctx.config
        needs = ctx.needs_input_grad
        direct = ctx.absolute.direct_buffer() if ctx.absolute is not None else None
        # the centre gradient doubles as dL/dmeans2d: written straight into
        # the view's block of means2d.grad when that block is untouched
        screen_direct = (ctx.screen_target.direct_buffer()
                         if needs[4] and ctx.screen_target is not None else None)
        gc, gq, ga, gb, absolute = stages.render_backward(
            stages.ProjectedFootprint(centers, conics),
            dict(ranges=ranges, point_list=ids, tile_order=order),
            colors, extras, True, background, final_t, contrib, g_features, cfg.width,
            cfg.height, absgrad=ctx.absolute is not None, constant_tail=1, need_a=needs[2],
            need_b=extras is not None and needs[3], gradient_alpha=g_alpha, separate_alpha=True,
            absolute_out=direct, centers_out=screen_direct)
        if ctx.absolute is not None and direct is None:
            ctx.absolute.write(absolute)
        g_screen = None
        if needs[4]:
            if ctx.screen_target is not None:
                if screen_direct is None:
                    ctx.screen_target.add(gc)  # into means2d.grad (see training.py)
            else:
                g_screen = gc
        return (gc if needs[0] else None, gq if needs[1] else None, ga, gb, g_screen, None, None,
                None, None, None, None, None, None, None)
