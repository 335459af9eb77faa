"""First-order autograd bridge for CUDA float32 SH0-3
(primitives/spherical_harmonics.py:1-159), backed by the sm_100a kernels."""

from __future__ import annotations

from numbers import Integral
from typing import Any

import torch
from torch import Tensor
from torch.autograd.function import once_differentiable

from . import stages


class _SphericalHarmonics(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, coefficients: Tensor, directions: Tensor, radii: Tensor | None,
                degree: int, grad_enabled: bool) -> Tensor:
        needs = (ctx.needs_input_grad[0], degree > 0 and ctx.needs_input_grad[1])
        save = grad_enabled and any(needs)
        colors, active = stages.sh_forward(coefficients, directions, degree, radii, save)
        if save:
            ctx.save_for_backward(coefficients, directions, radii, active)
            ctx.degree, ctx.needs = degree, needs
        ctx.set_materialize_grads(False)
        return colors

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, gradient: Tensor | None):
        if gradient is None:
            return (None,) * 5
        coefficients, directions, radii, active = ctx.saved_tensors
        need_coefficients, need_directions = ctx.needs
        grad_c, grad_d = stages.sh_backward(coefficients, directions, ctx.degree, radii, active,
                                            gradient, need_directions)
        return (grad_c if need_coefficients else None, grad_d if need_directions else None,
                None, None, None)


def spherical_harmonics(coefficients: Tensor, directions: Tensor, degree: int, *,
                        radii: Tensor | None = None) -> Tensor:
    """SH colour max(sum + 0.5, 0); rows with radii <= 0 return zero.

    Same validation and messages as primitives/spherical_harmonics.py:104-159.
    """
    if isinstance(degree, bool) or not isinstance(degree, Integral) or degree not in range(4):
        raise ValueError("SH degree must be an integer in [0,3]")
    if (not isinstance(coefficients, Tensor) or not coefficients.is_cuda
            or coefficients.dtype != torch.float32 or coefficients.ndim != 3
            or coefficients.shape[-1] != 3 or coefficients.shape[1] < (degree + 1) ** 2):
        raise ValueError("SH coefficients must be CUDA float32 (N,K,3) with enough coefficients")
    if (not isinstance(directions, Tensor) or directions.device != coefficients.device
            or directions.dtype != torch.float32 or directions.shape != (len(coefficients), 3)):
        raise ValueError("SH directions must be float32 (N,3) on the coefficients' device")
    if radii is not None and (radii.device != coefficients.device or radii.dtype != torch.int32
                              or radii.shape != (len(coefficients),)):
        raise ValueError("SH radii must be int32 (N,) on the coefficients' device")
    if degree == 0:
        directions = directions.detach()
    return _SphericalHarmonics.apply(coefficients, directions, radii, int(degree),
                                     torch.is_grad_enabled())
