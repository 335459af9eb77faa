"""Per-view densification metadata and auxiliary gradient targets
(dsl_splat/training.py:1-76, runtime/gradients.py:1-16)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
from torch import Tensor

from .inputs import Inputs


@dataclass(slots=True)
class AbsGradientTarget:
    """Destination of one view's |d means2d| sums (runtime/gradients.py:8-16)."""

    target: Tensor
    gaussian_ids: Tensor | None = None
    written: bool = False

    @torch.no_grad()
    def write(self, gradient: Tensor) -> None:
        value = gradient if self.gaussian_ids is None else gradient[self.gaussian_ids]
        self.target.copy_(value)
        self.written = True

    def direct_buffer(self) -> Tensor | None:
        """The target itself when a kernel may accumulate into it directly: a
        dense, contiguous view that still holds the zeros it was created with
        (the first backward through it).  Later backwards use write(), which
        replaces the values as the reference's copy does."""
        if self.written or self.gaussian_ids is not None or not self.target.is_contiguous():
            return None
        if self.target.dtype != torch.float32 or self.target.data_ptr() % 8:
            return None
        self.written = True
        return self.target


@dataclass(slots=True)
class ScreenGradientTarget:
    """Where one view's dL/dmeans2d lands in the means2d leaf's gradient.

    The reference routes it through autograd: each view's means2d is a
    select (dense) or an index_put + select (packed) of the leaf, whose
    backward materialises a zero-filled gradient of the whole (views, N, 2)
    leaf per view and then sums them -- O(views^2 N) work.  Here the render
    backward adds its centre gradient straight into the view's rows of
    leaf.grad (created zero-filled on first use): the view's (N, 2) block
    (dense), or its visible rows gathered by gaussian_ids (packed)."""

    leaf: Tensor
    index: int = 0                      # dense: view index into (views, N, 2)
    gaussian_ids: Tensor | None = None  # packed: this view's Gaussians, rows [begin, end)
    begin: int = 0
    end: int = 0
    # dense targets of one call share it: the gradient tensor this call
    # created and the views whose block of it is still untouched
    fresh: dict | None = None

    @torch.no_grad()
    def direct_buffer(self) -> Tensor | None:
        """Dense case: this view's (N, 2) block of leaf.grad when the block
        still holds the zeros this call created (the render backward then
        accumulates into it directly and add() is not needed), else None."""
        if self.gaussian_ids is not None or self.fresh is None:
            return None
        if self.leaf.grad is None:
            # zeros allocated beside absgrad's by the forward when it made both
            spare = self.fresh.pop("spare", None)
            self.leaf.grad = spare if spare is not None else torch.zeros_like(self.leaf)
            self.fresh["grad"] = self.leaf.grad
            self.fresh["views"] = set(range(self.fresh["count"]))
        if self.leaf.grad is not self.fresh.get("grad") or self.index not in self.fresh["views"]:
            return None
        # the view count is explicit: with N == 0 a -1 dimension is ambiguous
        block = self.leaf.grad.view(self.fresh["count"], *self.leaf.shape[-2:])[self.index]
        if not block.is_contiguous():
            return None
        self.fresh["views"].discard(self.index)
        return block

    @torch.no_grad()
    def add(self, gradient: Tensor) -> None:
        if self.leaf.grad is None:
            spare = self.fresh.pop("spare", None) if self.fresh is not None else None
            self.leaf.grad = spare if spare is not None else torch.zeros_like(self.leaf)
        if self.gaussian_ids is None:
            views = self.fresh["count"] if self.fresh is not None else -1
            self.leaf.grad.view(views, *gradient.shape)[self.index].add_(gradient)
        else:
            self.leaf.grad[self.begin:self.end].add_(gradient[self.gaussian_ids])


@dataclass(slots=True)
class TrainingMetadata:
    values: dict[str, Any]
    screen: Tensor | None
    absolute_targets: list[AbsGradientTarget | None]
    screen_targets: list[ScreenGradientTarget | None]


def prepare_training_metadata(dense: dict[str, Tensor], layout: Inputs, *, packed: bool,
                              absgrad: bool,
                              visible_counts: list[int] | None = None) -> TrainingMetadata:
    """training.py:24-76: dense or packed metadata, the means2d leaf and absgrad.

    visible_counts (packed): the per-view number of visible Gaussians, already
    read on the host (gs3d.rasterize reads them with the pair counts); the
    packed indices then come from nonzero_static and this function makes no
    host synchronisation of its own."""
    if packed:
        mask = (dense["radii"] > 0).all(-1)
        if visible_counts is None:
            batch_ids, camera_ids, gaussian_ids = mask.nonzero(as_tuple=True)
        else:
            idx = torch.nonzero_static(mask, size=int(sum(visible_counts)))
            batch_ids, camera_ids, gaussian_ids = idx.unbind(1)
        values = {name: v[batch_ids, camera_ids, gaussian_ids] for name, v in dense.items()}
    else:
        batch_ids = camera_ids = gaussian_ids = None
        values = {name: v.reshape(layout.batch_dims + tuple(v.shape[1:]))
                  for name, v in dense.items()}
    values.update(batch_ids=batch_ids, camera_ids=camera_ids, gaussian_ids=gaussian_ids)
    screen = values["means2d"].detach().requires_grad_(layout.requires_screen_grad)
    values["means2d"] = screen
    views = layout.batch_count * layout.cameras
    targets: list[AbsGradientTarget | None] = [None] * views
    if not layout.requires_screen_grad:
        return TrainingMetadata(values, None, targets, [None] * views)
    counts: list[int] | None = None
    if packed:
        if visible_counts is not None:
            counts = list(visible_counts)
        else:
            counts = ([len(screen)] if views == 1
                      else (dense["radii"] > 0).all(-1).sum(-1).flatten().tolist())
        screen_targets, begin = [], 0
        for count in counts:
            screen_targets.append(ScreenGradientTarget(
                screen, gaussian_ids=gaussian_ids[begin:begin + count], begin=begin,
                end=begin + count))
            begin += count
    else:
        fresh = {"count": views}
        screen_targets = [ScreenGradientTarget(screen, index=i, fresh=fresh)
                          for i in range(views)]
    if packed:
        dense_screen = torch.zeros_like(dense["means2d"]).index_put(
            (batch_ids, camera_ids, gaussian_ids), screen)
    else:
        dense_screen = screen.reshape(layout.batch_count, layout.cameras, layout.n, 2)
    if absgrad:
        if packed:
            absolute = torch.zeros_like(screen)
        else:
            # dense: absgrad and the first gradient of the means2d leaf come
            # from one zero fill (the leaf's gradient half is handed out by
            # the first direct_buffer() call of this call's views)
            pair = screen.new_zeros((2,) + tuple(screen.shape))
            absolute = pair[1]
            fresh["spare"] = pair[0]
        setattr(screen, "absgrad", absolute)
        if packed:
            begin = 0
            for i, count in enumerate(counts):
                end = begin + count
                targets[i] = AbsGradientTarget(absolute[begin:end], gaussian_ids[begin:end])
                begin = end
        else:
            views = absolute.reshape(layout.batch_count * layout.cameras, layout.n, 2)
            targets = [AbsGradientTarget(v) for v in views]
    return TrainingMetadata(values, dense_screen, targets, screen_targets)
