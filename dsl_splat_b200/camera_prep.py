"""GPU camera preparation and its pose VJP (splatting/cameras.py:1-175)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
from torch import Tensor
from torch.autograd.function import once_differentiable

from . import stages
from .cameras import PinholeCamera, validate_camera_options
from .inputs import check_tensor


@dataclass(frozen=True, slots=True)
class ViewConfig:
    width: int
    height: int
    near: float
    far: float
    radius_clip: float
    tile_mode: str = "radius"


class _PrepareCameras(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, views: Tensor, Ks: Tensor, width: int, height: int, grad_enabled: bool,
                with_centers: bool, status_sink: list | None = None):
        full, inverse, centers = stages.cameras_prepare(views, Ks, width, height, with_centers,
                                                        status_sink)
        if grad_enabled and ctx.needs_input_grad[0]:
            ctx.save_for_backward(Ks, inverse)
            ctx.width, ctx.height = width, height
            ctx.views_shape = views.shape
        ctx.set_materialize_grads(False)
        if not with_centers:
            ctx.mark_non_differentiable(centers)
        return full, centers

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, grad_full: Tensor | None, grad_centers: Tensor | None):
        if grad_full is None and grad_centers is None:
            return (None,) * 7
        Ks, inverse = ctx.saved_tensors
        grad_views = stages.cameras_backward(Ks, grad_full, ctx.width, ctx.height, inverse,
                                             grad_centers, ctx.views_shape)
        return grad_views, None, None, None, None, None, None


def _prepare(views, Ks, width, height, with_centers, status_sink=None):
    if torch.is_grad_enabled() and Ks.requires_grad:
        raise NotImplementedError("intrinsics gradients are not supported")
    return _PrepareCameras.apply(views, Ks, width, height, torch.is_grad_enabled(), with_centers,
                                 status_sink)


def prepare_cameras(views: Tensor, Ks: Tensor, width: int, height: int,
                    status_sink: list | None = None) -> Tensor:
    """Image-plane projection rows full = P V for every camera.

    status_sink defers the status read-back (see stages.cameras_prepare)."""
    return _prepare(views, Ks, width, height, False, status_sink)[0]


def prepare_cameras_with_centers(views: Tensor, Ks: Tensor, width: int, height: int,
                                 status_sink: list | None = None):
    """Projection rows and camera centres (for SH directions), one launch."""
    return _prepare(views, Ks, width, height, True, status_sink)


def prepare_camera(camera: PinholeCamera, radius_clip: float):
    """splatting/cameras.py:147-175 for the stage-level API."""
    validate_camera_options(camera.width, camera.height, camera.near_plane, camera.far_plane,
                            radius_clip)
    if not isinstance(camera.viewmat, Tensor) or not camera.viewmat.is_cuda:
        raise ValueError("camera tensors must be CUDA float32")
    check_tensor("viewmat", camera.viewmat, camera.viewmat.device, (4, 4))
    check_tensor("K", camera.K, camera.viewmat.device, (3, 3))
    if torch.is_grad_enabled() and camera.K.requires_grad:
        raise NotImplementedError("intrinsics gradients are not supported")
    intrinsic = camera.K.detach().contiguous()
    view = camera.viewmat.contiguous()
    projection = prepare_cameras(view, intrinsic, camera.width, camera.height)
    config = ViewConfig(camera.width, camera.height, camera.near_plane, camera.far_plane,
                        radius_clip)
    return view, projection, intrinsic, config
