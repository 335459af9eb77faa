"""Batched Gaussian layouts and input checks (dsl_splat/inputs.py:1-269).

The host side of the drop-in: same shapes, batching rules, error messages
and quaternion normalisation (a Torch op, as in the reference) before the
CUDA stages run.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Literal

import torch
import torch.nn.functional as F
from torch import Tensor

RenderMode = Literal["RGB", "D", "ED", "RGB+D", "RGB+ED"]


def batch_item(values: Tensor, index: int) -> Tensor:
    """Singleton batches use squeeze (a view without a gradient scatter)."""
    return values.squeeze(0) if index == 0 and values.shape[0] == 1 else values[index]


@dataclass(slots=True)
class ViewFeatures:
    values: tuple[Tensor, ...]
    per_view: bool

    @property
    def channels(self) -> int:
        return self.values[0].shape[-1]

    def at(self, batch: int, camera: int) -> Tensor:
        v = self.values[batch]
        return batch_item(v, camera) if self.per_view else v


@dataclass(slots=True)
class Inputs:
    batch_dims: tuple[int, ...]
    batch_count: int
    n: int
    cameras: int
    device: torch.device
    means: tuple[Tensor, ...]
    quats: tuple[Tensor, ...]
    scales: tuple[Tensor, ...]
    opacities: tuple[Tensor, ...]
    viewmats: Tensor
    Ks: Tensor
    colors: ViewFeatures
    backgrounds: Tensor | None
    extras: ViewFeatures | None
    filters: Tensor | None
    requires_screen_grad: bool


def check_tensor(name: str, tensor, device, shape=None) -> None:
    if not isinstance(tensor, Tensor) or tensor.device != device or tensor.dtype != torch.float32:
        raise ValueError(f"{name} must be float32 on {device}")
    if shape is not None and tuple(tensor.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(tensor.shape)}")


def _batch_views(value: Tensor, batch_count: int, item_shape: tuple[int, ...]):
    if batch_count == 1:
        return (value if value.shape == item_shape else value.reshape(item_shape),)
    shape = (batch_count,) + item_shape
    return (value if value.shape == shape else value.reshape(shape)).unbind(0)


def _view_values(name, value, batch_dims, batch_count, cameras, n, device, *, sh=False):
    check_tensor(name, value, device)
    trailing = 3 if sh else 2
    shared_rank = len(batch_dims) + trailing
    per_view = value.ndim == shared_rank + 1
    tail = tuple(value.shape[-trailing:])
    expected = batch_dims + ((cameras,) if per_view else ()) + tail
    if (value.ndim not in (shared_rank, shared_rank + 1) or tuple(value.shape) != expected
            or tail[0] != n or tail[-1] <= 0):
        raise ValueError(
            f"{name} must have batch dimensions {batch_dims} and shape (...,N,D) or (...,C,N,D)"
            if not sh else f"{name} must be (...,N,K,3) or (...,C,N,K,3)")
    if sh and tail[-1] != 3:
        raise ValueError("SH colors must have three channels")
    item_shape = ((cameras,) if per_view else ()) + tail
    return ViewFeatures(_batch_views(value, batch_count, item_shape), per_view)


def normalize_inputs(means, quats, scales, opacities, colors, viewmats, Ks, backgrounds, extras,
                     filter3D, sh_degree, *, normalize_quats: bool = True) -> Inputs:
    """inputs.py:164-269: layout checks, per-batch views, normalised quats."""
    if not isinstance(means, Tensor) or not means.is_cuda or means.ndim < 2 or means.shape[-1] != 3:
        raise ValueError("means must be a CUDA float32 tensor with shape (...,N,3)")
    device = means.device
    check_tensor("means", means, device)
    batch_dims = tuple(means.shape[:-2])
    batch_count, n = math.prod(batch_dims), means.shape[-2]
    if batch_count <= 0:
        raise ValueError("Gaussian batch dimensions must be nonempty")
    check_tensor("quats", quats, device, batch_dims + (n, 4))
    check_tensor("scales", scales, device, batch_dims + (n, 3))
    check_tensor("opacities", opacities, device, batch_dims + (n,))
    check_tensor("viewmats", viewmats, device)
    if (viewmats.ndim != len(batch_dims) + 3 or viewmats.shape[-2:] != (4, 4)
            or tuple(viewmats.shape[:-3]) != batch_dims):
        raise ValueError("viewmats must have shape (...,C,4,4) with the Gaussian batch dimensions")
    cameras = viewmats.shape[-3]
    if cameras <= 0:
        raise ValueError("at least one camera is required")
    check_tensor("Ks", Ks, device, batch_dims + (cameras, 3, 3))
    if colors is None:
        raise ValueError("colors is required for RGB/features rendering")
    bank = _view_values("colors", colors, batch_dims, batch_count, cameras, n, device,
                        sh=sh_degree is not None)
    if sh_degree is not None and bank.values[0].shape[-2] < (sh_degree + 1) ** 2:
        raise ValueError("not enough SH coefficients for sh_degree")
    d = bank.channels
    bg = None
    if backgrounds is not None:
        check_tensor("backgrounds", backgrounds, device, batch_dims + (cameras, d))
        bg = backgrounds.reshape(batch_count, cameras, d)
    extra_bank = None
    if extras is not None:
        extra_bank = _view_values("extra_signals", extras, batch_dims, batch_count, cameras, n,
                                  device)
    filters = None
    if filter3D is not None:
        check_tensor("filter3D", filter3D, device)
        if tuple(filter3D.shape) not in (batch_dims + (n,), batch_dims + (n, 1)):
            raise ValueError("filter3D must have shape (...,N) or (...,N,1)")
        filters = filter3D.reshape(batch_count, n)
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (Ks, backgrounds)):
        raise NotImplementedError("intrinsics/background gradients are not supported")
    return Inputs(
        batch_dims, batch_count, n, cameras, device,
        _batch_views(means, batch_count, (n, 3)),
        _batch_views(F.normalize(quats, dim=-1) if normalize_quats else quats, batch_count, (n, 4)),
        _batch_views(scales, batch_count, (n, 3)),
        _batch_views(opacities, batch_count, (n,)),
        viewmats.reshape(batch_count, cameras, 4, 4),
        Ks.detach().reshape(batch_count, cameras, 3, 3),
        bank, bg, extra_bank, filters,
        torch.is_grad_enabled() and any(
            isinstance(v, Tensor) and v.requires_grad
            for v in (means, quats, scales, opacities, colors, extras, viewmats)),
    )


def spherical_harmonics(coefficients: Tensor, directions: Tensor, degree: int) -> Tensor:
    """inputs.py:54-60 on the CUDA SH kernel.  The reference's Torch branch
    for CPU / float64 callers has no counterpart: this library has no CPU
    compute path, so other inputs are rejected."""
    if not (coefficients.is_cuda and coefficients.dtype == directions.dtype == torch.float32):
        raise ValueError("spherical_harmonics needs CUDA float32 coefficients and directions")
    from .spherical_harmonics import spherical_harmonics as cuda_sh
    return cuda_sh(coefficients, directions, degree)
