"""Camera-sharded data parallelism for multi-view gs3d training.

dsl_splat renders the views of a batch one after another and lets autograd
sum their per-Gaussian gradients (gs3d/api.py:132-189, 229-255).  Across
GPUs the same sum is an all-reduce: every rank holds the full Gaussian set,
renders the cameras {k : k mod world == rank}, runs its backward (which
already sums its local views), and the ranks all-reduce the per-Gaussian
gradients (means 3 + quats 4 + scales 3 + opacities 1 + SH 48 floats per
Gaussian).  That all-reduce is the path's only exchange; images, means2d
gradients and pose gradients stay on the rank that rendered them.

Two ways to run the exchange:

* `allreduce_parameter_grads` after `backward()` (one coalesced all-reduce);
* `GradientSync`, a context around the rasterize + backward calls: every
  local view's projection backward accumulates straight into one gradient
  buffer per parameter (no per-view gradient tensors, no autograd sums), and
  the last local view runs its projection backward in Gaussian-range buckets,
  issuing each bucket's all-reduce as soon as its kernel is queued, so the
  NCCL transfer of bucket b overlaps the kernel of bucket b+1 (NCCL runs on
  its own stream, ordered after the work queued before the call).

Works with any torch.distributed backend (NCCL over NVLink on the GPUs,
gloo for the CPU tests).
"""

from __future__ import annotations

import threading
from datetime import timedelta
from typing import Sequence

import torch
import torch.distributed as dist
from torch import Tensor

_ACTIVE = threading.local()


def local_cameras(cameras: int, rank: int, world: int) -> list[int]:
    """Camera indices rank renders: k mod world == rank (round robin)."""
    if not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    return list(range(rank, cameras, world))


def shard_views(viewmats: Tensor, Ks: Tensor, rank: int, world: int) -> tuple[Tensor, Tensor, list[int]]:
    """The (C_local,4,4) poses and (C_local,3,3) intrinsics of this rank."""
    idx = local_cameras(viewmats.shape[-3], rank, world)
    sel = torch.tensor(idx, dtype=torch.long, device=viewmats.device)
    return viewmats.index_select(-3, sel), Ks.index_select(-3, sel), idx


def allreduce_gradients(grads: Sequence[Tensor | None], group=None) -> None:
    """Sum gradients over all ranks in place.

    On NCCL the all-reduces are issued as one coalesced group (one launch,
    like a single flat buffer: 0.47 ms instead of 0.57 ms for the config-1
    gradient set on two B200s, with no copy into a flat buffer); other
    backends get one async all-reduce per tensor.  Ranks must pass the same
    sequence (None entries are skipped on every rank alike, so the
    collectives line up).
    """
    tensors = [g for g in grads if g is not None]
    if not tensors:
        return
    backend = dist.get_backend(group)
    if backend == "nccl" and len(tensors) > 1 and hasattr(dist, "_coalescing_manager"):
        with dist._coalescing_manager(group=group, async_ops=True) as cm:
            for g in tensors:
                dist.all_reduce(g, op=dist.ReduceOp.SUM, group=group)
        cm.wait()
        return
    handles = [dist.all_reduce(g, op=dist.ReduceOp.SUM, group=group, async_op=True)
               for g in tensors]
    for h in handles:
        h.wait()


def allreduce_parameter_grads(params: Sequence[Tensor], group=None) -> None:
    """all-reduce p.grad of every parameter that requires a gradient.

    A rank whose backward produced no gradient for a parameter (it rendered
    no view: fewer cameras than ranks) contributes zeros, so every rank
    issues the same collectives in the same order."""
    grads = []
    for p in params:
        if not p.requires_grad:
            continue
        if p.grad is None:
            p.grad = torch.zeros_like(p)
        grads.append(p.grad)
    allreduce_gradients(grads, group=group)


def init_process_group(backend: str, timeout_s: float = 120.0, device: torch.device | None = None):
    """Process group from the torchrun environment with a short timeout, so a
    rank that stops joining collectives ends the others' next collective with
    an error instead of a hang."""
    kw = {"timeout": timedelta(seconds=timeout_s)}
    if device is not None and device.type == "cuda":
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)
    return dist.group.WORLD


def bucket_bounds(n: int, buckets: int, align: int = 32) -> list[tuple[int, int]]:
    """[lo, hi) Gaussian ranges covering [0, n): at most `buckets` of them,
    inner boundaries on multiples of `align` (the projection backward's chunk
    of 32, which keeps every row pointer of a bucket 16-byte aligned)."""
    if n <= 0:
        return []
    if buckets < 1 or align < 1:
        raise ValueError("buckets and align must be positive")
    step = -(-n // buckets)
    step = -(-step // align) * align
    return [(lo, min(lo + step, n)) for lo in range(0, n, step)]


def current_sync() -> "GradientSync | None":
    """The GradientSync context active on this thread, if any."""
    return getattr(_ACTIVE, "sync", None)


class GradientSync:
    """Per-Gaussian gradient exchange overlapped with the projection backward.

    Usage (one rank per GPU, the same calls on every rank)::

        sync = GradientSync(means, quats, scales, opacities, sh, group=pg)
        with sync:
            res = gs3d.rasterize(means, quats, scales, opacities, views, Ks, W, H,
                                 sh_coeffs=sh)
            torch.autograd.backward(...)
        sync.wait()   # p.grad now holds the sum over every rank's views

    Inside the context, gs3d.rasterize calls whose Gaussian tensors are these
    leaves (same storage and shape, no batch dimensions) send their
    per-Gaussian gradients here instead of through autograd: each local view
    accumulates into one buffer per parameter, and the last local view's
    backward launches in `buckets` Gaussian ranges, each followed by the
    asynchronous all-reduce of its slices.  `wait()` orders the current
    stream after the reductions and publishes the buffers as p.grad (added to
    an existing p.grad, as autograd accumulates: only this step's gradient is
    reduced).  Gradients of other
    inputs (poses, means2d) are unaffected, and calls that do not match the
    leaves fall back to autograd.  With group=None nothing is reduced: the
    context still saves the per-view gradient tensors.

    buckets=1 issues one all-reduce of one flat buffer (the per-parameter
    buffers are views of it) after the last kernel; more buckets all-reduce
    row ranges of every buffer as coalesced groups, overlapping the transfers
    with the remaining kernels.  On two B200s
    (config 1, 236 MB of gradients) one bucket measured fastest: NCCL's
    kernels and the projection backward contend for SMs and HBM (762 / 733 /
    722 / 668 frames/s for 1 / 2 / 4 / 8 buckets).
    """

    NAMES = ("means", "quats", "scales", "opacities", "sh")

    def __init__(self, means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor,
                 sh: Tensor | None = None, *, group=None, buckets: int = 1):
        self.params = dict(zip(self.NAMES, (means, quats, scales, opacities, sh)))
        self.group = group
        self.buckets = buckets
        self._reset()

    def _reset(self):
        self.views = 0
        self.done = 0
        self.buffers: dict[str, Tensor] | None = None
        self.flat: Tensor | None = None
        self.works: list = []
        self.finished = False

    def __enter__(self) -> "GradientSync":
        if current_sync() is not None:
            raise RuntimeError("GradientSync contexts do not nest")
        self._reset()
        _ACTIVE.sync = self
        return self

    def __exit__(self, *exc) -> None:
        _ACTIVE.sync = None

    # ---- called by the projection autograd node -------------------------------
    def claims(self, means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor,
               sh: Tensor | None) -> bool:
        """True when these projection inputs are the registered leaves."""
        for name, t in zip(self.NAMES, (means, quats, scales, opacities, sh)):
            leaf = self.params[name]
            if (t is None) != (leaf is None):
                return False
            if t is not None and (t.data_ptr() != leaf.data_ptr() or t.shape != leaf.shape
                                  or not t.is_contiguous()):
                return False
        return True

    def register_view(self) -> None:
        self.views += 1

    def begin_view(self) -> tuple[dict[str, Tensor], bool, bool]:
        """Buffers for the next view's backward, its accumulate flag, and
        whether it is the last local view (the one that reduces)."""
        self._make_buffers()
        accumulate = self.done > 0  # the first view's backward overwrites
        self.done += 1
        return self.buffers, accumulate, self.done == self.views

    def _make_buffers(self) -> None:
        if self.buffers is None:
            # views of one flat allocation: a bucket covering every row is then
            # one all-reduce of one buffer (0.60 ms instead of 0.82 ms for a
            # coalesced group of the five tensors, 236 MB on 4 B200s)
            live = {k: p for k, p in self.params.items() if p is not None and p.requires_grad}
            same = len({(p.dtype, p.device) for p in live.values()}) == 1
            if live and same:
                first = next(iter(live.values()))
                self.flat = torch.empty(sum(p.numel() for p in live.values()),
                                        dtype=first.dtype, device=first.device)
                self.buffers, at = {}, 0
                for k, p in live.items():
                    self.buffers[k] = self.flat[at:at + p.numel()].view(p.shape)
                    at += p.numel()
            else:
                self.flat = None
                self.buffers = {k: torch.empty_like(p) for k, p in live.items()}

    def reduce_range(self, lo: int, hi: int) -> None:
        """Issue the all-reduce of rows [lo, hi) of every buffer (async)."""
        if self.group is None:
            return
        rows = {len(b) for b in self.buffers.values()}
        if self.flat is not None and lo == 0 and rows == {hi}:
            self.works.append(dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=self.group,
                                              async_op=True))
            return
        tensors = [b[lo:hi] for b in self.buffers.values()]
        if dist.get_backend(self.group) == "nccl" and hasattr(dist, "_coalescing_manager"):
            with dist._coalescing_manager(group=self.group, async_ops=True) as cm:
                for t in tensors:
                    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
            self.works.append(cm)
        else:
            self.works.extend(dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group,
                                              async_op=True) for t in tensors)

    def finish(self) -> None:
        self.finished = True

    def wait(self) -> None:
        """Order the current stream after the reductions; publish p.grad."""
        if self.views and not self.finished:
            raise RuntimeError(f"GradientSync: {self.done} of {self.views} view backwards ran")
        if self.group is not None and self.views == 0 and not self.works:
            # this rank rendered no view (fewer cameras than ranks): it joins
            # the other ranks' all-reduces with zero gradients, bucket for
            # bucket as their last view's backward issues them
            self._make_buffers()
            for buf in self.buffers.values():
                buf.zero_()
            n = self.params["means"].shape[0]
            for lo, hi in bucket_bounds(n, self.buckets):
                self.reduce_range(lo, hi)
        for w in self.works:
            w.wait()
        self.works = []
        for name, buf in (self.buffers or {}).items():
            p = self.params[name]
            if p.grad is None:
                p.grad = buf
            elif p.grad is not buf:
                p.grad.add_(buf)
