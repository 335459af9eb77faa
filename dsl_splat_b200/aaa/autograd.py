"""First-order autograd bridge of one AAA view (aaa/autograd.py:34-235).

Forward: the HIER blend of the view's preprocessed and binned Gaussians
(preprocessing and binning ran before, as aaa/frame.py prepares the frame
outside the reference's Function).  Backward: the replay gives the
transform, opacity, feature and screen gradients; the preprocessing adjoint
maps them to means, scales, quaternions and opacities, and the camera
adjoint to the lowered camera tensors, whose Torch lowering carries them on
to viewmats.
"""

from __future__ import annotations

from typing import Any

import torch
from torch.autograd.function import once_differentiable

from . import stages


class RasterizeView(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, means, quats, scales, opacities, features, means2d, viewmatrix,
                projmatrix, campos, view: stages.AaaView, settings, state: stages.AaaState,
                bins: dict, background, filters, absgrad_target, grad_enabled: bool,
                statistics=None):
        cull = bool(settings.culling_settings.hierarchical_4x4_culling)
        features = features.contiguous()
        needs_backward = grad_enabled and any(ctx.needs_input_grad[:9])
        # a forward that will be differentiated keeps its blend records, so
        # the backward reads each pixel's samples instead of replaying queues
        image, final_t, contrib, records = stages.render(
            state, bins, features, background, view.width, view.height, cull,
            record_capacity=stages.RECORD_CAPACITY if needs_backward else 0,
            statistics=statistics)
        if means.shape[0] == 0:
            image.zero_()
        ctx.mark_non_differentiable(final_t, contrib)
        ctx.set_materialize_grads(False)
        if not needs_backward:
            return image, final_t, contrib
        ctx.save_for_backward(means, quats, scales, opacities, features, image, final_t,
                              background)
        ctx.view, ctx.settings, ctx.state, ctx.bins, ctx.cull = view, settings, state, bins, cull
        ctx.records = records
        ctx.filters = filters
        ctx.screen = means2d is not None
        ctx.absgrad_target = absgrad_target
        return image, final_t, contrib

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, grad_image, grad_t, grad_contrib):
        none = (None,) * 18
        if grad_image is None:
            return none
        means, quats, scales, opacities, features, image, final_t, background = ctx.saved_tensors
        view, st = ctx.view, ctx.state
        absgrad = ctx.absgrad_target is not None
        g_tr, g_op, g_col, g_scr, g_abs = stages.render_backward(
            st, ctx.bins, features, background, image, final_t, grad_image.contiguous(),
            view.width, view.height, ctx.cull, screen=ctx.screen, absgrad=absgrad,
            records=ctx.records)
        if absgrad:
            ctx.absgrad_target.write(g_abs)
        needs = ctx.needs_input_grad
        g_means = g_quats = g_scales = g_opac = None
        if any(needs[:4]):
            g_opac, g_means, g_scales, g_quats = stages.preprocess_backward(
                view, ctx.settings, means, quats, scales, opacities, st, g_tr, g_op)
        g_view = g_proj = g_campos = None
        if any(needs[6:9]):
            g_view, g_proj, g_campos = stages.camera_backward(
                view, ctx.settings, means, quats, scales, ctx.filters, st, g_tr, g_op)
        return (g_means if needs[0] else None, g_quats if needs[1] else None,
                g_scales if needs[2] else None,
                g_opac.reshape_as(opacities) if needs[3] else None,
                g_col if needs[4] else None, g_scr if needs[5] and g_scr is not None else None,
                g_view if needs[6] else None, g_proj if needs[7] else None,
                g_campos if needs[8] else None) + (None,) * 9


__all__ = ["RasterizeView"]
