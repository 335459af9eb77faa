"""Contribution statistics requests (dsl_splat/statistics.py:1-156).

Masks and weights only affect the statistics, never the image.  Each request
returns (..., cameras, N) values owned by the render call.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch
from torch import Tensor


@dataclass(frozen=True, slots=True)
class MaskedContributionCount:
    name: str
    mask: Tensor


@dataclass(frozen=True, slots=True)
class WeightedContributionSum:
    name: str
    pixel_weights: Tensor


StatisticsRequest = MaskedContributionCount | WeightedContributionSum
StatisticsKey = tuple[int, ...]


@dataclass(slots=True)
class PreparedStatistics:
    key: StatisticsKey        # per request: 0 = masked count, 1 = weighted sum
    pixel_values: Tensor      # (R, H*W) float32
    counts: Tensor            # (Rc, N) int32
    sums: Tensor              # (Rs, N) float32


def prepare_statistics(requests: Sequence[StatisticsRequest], *, batch_dims, batch_count,
                       cameras, n, width, height, device):
    """statistics.py:75-153: validate maps, allocate (…,C,N) outputs."""
    names: set[str] = set()
    maps: list[Tensor] = []
    kinds: list[int] = []
    shape = tuple(batch_dims) + (cameras, height, width)
    for request in requests:
        if not isinstance(request, (MaskedContributionCount, WeightedContributionSum)):
            raise TypeError("unsupported contribution statistics request")
        if not isinstance(request.name, str) or not request.name or request.name in names:
            raise ValueError("statistics names must be nonempty and unique")
        names.add(request.name)
        count = isinstance(request, MaskedContributionCount)
        value = request.mask if count else request.pixel_weights
        dtype = torch.bool if count else torch.float32
        if not isinstance(value, Tensor) or value.device != device or value.dtype != dtype:
            raise ValueError(f"statistics {request.name!r} must use {dtype} on {device}")
        if value.requires_grad:
            raise ValueError("statistics pixel maps are non-differentiable constants")
        if tuple(value.shape) == (height, width):
            value = value.expand(batch_count, cameras, height, width)
        elif tuple(value.shape) == shape:
            value = value.reshape(batch_count, cameras, height, width)
        else:
            raise ValueError(f"statistics maps must have shape {(height, width)} or {shape}")
        maps.append(value.to(torch.float32))
        kinds.append(0 if count else 1)
    key = tuple(kinds)
    pixel_values = torch.stack(maps, dim=2).reshape(batch_count, cameras, len(maps), -1)
    counts = torch.zeros((batch_count, cameras, kinds.count(0), n), dtype=torch.int32, device=device)
    sums = torch.zeros((batch_count, cameras, kinds.count(1), n), dtype=torch.float32, device=device)
    destinations = {0: counts, 1: sums}
    results = {
        request.name: destinations[kinds[i]][:, :, sum(k == kinds[i] for k in kinds[:i])].view(
            tuple(batch_dims) + (cameras, n))
        for i, request in enumerate(requests)
    }
    prepared = [PreparedStatistics(key, pixel_values[b, c].contiguous(), counts[b, c], sums[b, c])
                for b in range(batch_count) for c in range(cameras)]
    return prepared, results


__all__ = ["MaskedContributionCount", "WeightedContributionSum", "StatisticsRequest"]
