"""Explicit Mip-style 3D filtering used by the official RaDe-GS frontend
(rade/filtering.py:7-26): plain Torch, ordinary gradients."""

from __future__ import annotations

from torch import Tensor


def apply_3d_filter(scales: Tensor, opacities: Tensor, filter_3d: Tensor) -> tuple[Tensor, Tensor]:
    """Filtered scales sqrt(s^2 + f^2) and opacities times
    sqrt(prod s^2 / prod (s^2 + f^2)).

    scales: (...,N,3), opacities: (...,N), filter_3d: (...,N,1).
    """
    if filter_3d.shape != scales.shape[:-1] + (1,) or opacities.shape != scales.shape[:-1]:
        raise ValueError("require scales (...,N,3), opacities (...,N), filter_3d (...,N,1)")
    squares = scales.square()
    filtered = squares + filter_3d.square()
    coefficient = (squares.prod(-1) / filtered.prod(-1)).sqrt()
    return filtered.sqrt(), opacities * coefficient
