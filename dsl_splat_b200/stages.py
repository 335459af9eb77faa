"""Stage wrappers: allocate outputs with Torch and launch one C-ABI call.

These are the swap points of the reference's L2 stage wrappers:
gs3d/projection.py:309-428 (prepare/backward), splatting/binning.py:72-117
(bin_and_sort), gs3d/render.py:359-463 (render/backward),
primitives/spherical_harmonics.py:18-101, splatting/cameras.py:27-115 and
splatting/metadata.py:34-70.  Everything runs on the caller's current CUDA
stream; tensors must be CUDA float32/int32.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch
from torch import Tensor

from . import _native as nv
from ._native import check, lib, ptr


def _stream(t: Tensor) -> int:
    return nv.stream(t.device)


# Optional per-stage CUDA-event timing: when TIMERS is a dict, the wrapped
# stages record (start, end) event pairs on the launching stream under their
# name.  bench.py uses this to time the dominant kernel live.
TIMERS: dict[str, list] | None = None


class _timed:
    __slots__ = ("name", "device", "start")

    def __init__(self, name: str, device: torch.device):
        self.name, self.device = name, device

    def __enter__(self):
        if TIMERS is not None:
            self.start = torch.cuda.Event(enable_timing=True)
            self.start.record(torch.cuda.current_stream(self.device))
        return self

    def __exit__(self, *exc):
        if TIMERS is not None:
            end = torch.cuda.Event(enable_timing=True)
            end.record(torch.cuda.current_stream(self.device))
            TIMERS.setdefault(self.name, []).append((self.start, end))
        return False


def _c(t: Tensor | None) -> Tensor | None:
    """Contiguous, with a 16-byte-aligned base (the kernels load float2/float4 rows)."""
    if t is None:
        return None
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


class Args:
    """Converts tensors to device addresses for one C call and keeps every
    converted tensor referenced until the call has been enqueued.

    A copy made only to pass its address (a contiguous or aligned clone)
    would otherwise be freed at once, and the caching allocator could hand
    its block to the next argument's copy before the kernel reads it.
    """

    __slots__ = ("keep",)

    def __init__(self):
        self.keep: list[Tensor] = []

    def __call__(self, t: Tensor | None) -> int | None:
        if t is None:
            return None
        t = _c(t)
        self.keep.append(t)
        return t.data_ptr()


def _far(value: float) -> float:
    return float(value) if math.isfinite(value) else float("inf")


@dataclass(slots=True)
class ProjectedFootprint:
    centers: Tensor
    conics: Tensor


@dataclass(slots=True)
class ProjectedGaussians(ProjectedFootprint):
    radii: Tensor
    tile_counts: Tensor
    depths: Tensor


@dataclass(slots=True)
class RenderedPixels:
    features: Tensor       # (H, W, C') interleaved, or (C', H, W) planar
    transmittance: Tensor  # (H, W)
    contributors: Tensor   # (H, W) int32
    alpha: Tensor | None = None  # (H, W, 1) when rendered apart (features then hold C'-1)


# ---- cameras ---------------------------------------------------------------

def raise_camera_errors(codes) -> None:
    """splatting/cameras.py:64-74: the reference's exceptions for status codes."""
    if 2 in codes:
        raise ValueError("Ks must be finite with positive fx/fy")
    if 1 in codes:
        raise NotImplementedError("Ks must be a zero-skew pinhole intrinsic matrix")
    if 3 in codes:
        raise torch.linalg.LinAlgError("viewmats must be invertible for SH directions")


def cameras_prepare(views: Tensor, Ks: Tensor, width: int, height: int, with_centers: bool,
                    status_sink: list | None = None):
    """splatting/cameras.py:29-85: full (…,4,4), inverse (C,4,4), centers (…,3).

    Only status codes cross to the host, as in the reference.  With a
    status_sink the (C,) int32 codes are appended to it instead of being read
    now, so the caller can fold that read into its next host synchronisation
    (bin_and_sort_many does) and raise the same exceptions there."""
    views_c, Ks_c = views.reshape(-1, 4, 4).contiguous(), Ks.reshape(-1, 3, 3).contiguous()
    count = len(views_c)
    full = torch.empty(views.shape, dtype=torch.float32, device=views.device)
    inverse = views.new_empty((count if with_centers else 0, 4, 4))
    centers = views.new_empty(views.shape[:-2] + (3,) if with_centers else (0, 3))
    errors = torch.empty(count, dtype=torch.int32, device=views.device)
    check(lib.splat_cameras_prepare(count, ptr(views_c), ptr(Ks_c), width, height, int(with_centers),
                                    ptr(full), ptr(inverse) if with_centers else None,
                                    ptr(centers) if with_centers else None, ptr(errors),
                                    _stream(views)), "cameras_prepare")
    if status_sink is not None:
        status_sink.append(errors)
    else:
        raise_camera_errors(errors.tolist())
    return full, inverse, centers


def cameras_backward(Ks: Tensor, grad_full: Tensor | None, width: int, height: int,
                     inverse: Tensor, grad_centers: Tensor | None, views_shape) -> Tensor:
    Ks_c = Ks.reshape(-1, 3, 3).contiguous()
    count = len(Ks_c)
    grad_views = torch.empty(views_shape, dtype=torch.float32, device=Ks.device)
    gf = None if grad_full is None else grad_full.reshape(-1, 4, 4).contiguous()
    gc = None if grad_centers is None else grad_centers.reshape(-1, 3).contiguous()
    check(lib.splat_cameras_backward(count, ptr(Ks_c), ptr(gf), width, height,
                                     ptr(inverse) if gc is not None else None, ptr(gc),
                                     ptr(grad_views), _stream(Ks)), "cameras_backward")
    return grad_views


# ---- projection --------------------------------------------------------------

TILE_MODES = {"radius": 0, "snugbox": 1, "accutile": 2}


def _tile_mode(mode: str) -> int:
    """splatting/intersections.py:24-26 validate_tile_mode, as the C code."""
    if mode not in TILE_MODES:
        raise ValueError("tile_mode must be 'radius', 'snugbox' or 'accutile'")
    return TILE_MODES[mode]


def project(means, quats, scales, opacities, view, projection, intrinsics, width, height,
            near, far, radius_clip, tile_mode: str = "radius") -> ProjectedGaussians:
    """gs3d/projection.py:309-354 prepare (tile counts of tile_mode)."""
    pin = Args()
    n = len(means)
    state = ProjectedGaussians(means.new_empty((n, 2)), means.new_empty((n, 4)),
                               torch.empty(n, dtype=torch.int32, device=means.device),
                               torch.empty(n, dtype=torch.int32, device=means.device),
                               means.new_empty(n))
    if n:
        check(lib.splat_project_forward(
            n, pin(means), pin(quats), pin(scales), pin(opacities),
            pin(view), pin(projection), pin(intrinsics), width, height, float(near),
            _far(far), float(radius_clip), ptr(state.centers), ptr(state.conics),
            ptr(state.radii), ptr(state.tile_counts), ptr(state.depths), _tile_mode(tile_mode),
            _stream(means)), "project_forward")
    return state


@dataclass(slots=True)
class FusedProjection:
    state: ProjectedGaussians
    colors: Tensor | None      # (n,3) SH colours
    active: Tensor | None      # (n,3) uint8
    means2d: Tensor
    opacities: Tensor
    conics3: Tensor


def project_fused(means, quats, scales, opacities, view, projection, intrinsics, width, height,
                  near, far, radius_clip, sh: Tensor | None = None, sh_degree: int = 0,
                  campos: Tensor | None = None, need_active: bool = True,
                  normalize_quats: bool = False, tile_mode: str = "radius") -> FusedProjection:
    """One launch for gs3d/api.py:145-189: projection, masked SH and metadata.

    normalize_quats: quats are raw; the kernel applies F.normalize with the
    bits of Torch's CUDA implementation (inputs.py:252)."""
    pin = Args()
    n = len(means)
    dev = means.device
    state = ProjectedGaussians(means.new_empty((n, 2)), means.new_empty((n, 4)),
                               torch.empty(n, dtype=torch.int32, device=dev),
                               torch.empty(n, dtype=torch.int32, device=dev), means.new_empty(n))
    colors = means.new_empty((n, 3)) if sh is not None else None
    active = (torch.empty((n, 3), dtype=torch.uint8, device=dev)
              if sh is not None and need_active else None)
    m2d, mop, mcon = means.new_empty((n, 2)), means.new_empty(n), means.new_empty((n, 3))
    if n:
        sh_c = _c(sh)
        check(lib.splat_project_forward_fused(
            n, pin(means), pin(quats), int(normalize_quats), pin(scales), pin(opacities),
            pin(view), pin(projection), pin(intrinsics), width, height, float(near),
            _far(far), float(radius_clip), ptr(state.centers), ptr(state.conics),
            ptr(state.radii), ptr(state.tile_counts), ptr(state.depths), int(sh_degree),
            sh_c.shape[1] if sh_c is not None else 0, ptr(sh_c), pin(campos), ptr(colors), 3,
            ptr(active), ptr(m2d), ptr(mop), ptr(mcon), _tile_mode(tile_mode), _stream(means)),
            "project_forward_fused")
    return FusedProjection(state, colors, active, m2d, mop, mcon)


@dataclass(slots=True)
class ViewsProjection:
    """project_views outputs: per-view tensors for the differentiable
    outputs, stacked (views, n, ...) tensors for the rest."""
    centers: list[Tensor]        # views x (n,2)
    conics: list[Tensor]         # views x (n,4)
    colors: list[Tensor] | None  # views x (n,3)
    radii: Tensor                # (views,n) int32
    tile_counts: Tensor          # (views,n) int32
    depths: Tensor               # (views,n)
    active: Tensor | None        # (views,n,3) uint8
    means2d: Tensor              # (views,n,2)
    opacities: Tensor            # (views,n)
    conics3: Tensor              # (views,n,3)

    def state(self, v: int) -> ProjectedGaussians:
        return ProjectedGaussians(self.centers[v], self.conics[v], self.radii[v],
                                  self.tile_counts[v], self.depths[v])


def pointer_table(tensors) -> ctypes.Array:
    """Host array of device addresses (one per view) for the C ABI."""
    tensors = list(tensors)
    return (ctypes.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])


def project_views(means, quats, scales, opacities, views, projections, intrinsics, width,
                  height, near, far, radius_clip, sh: Tensor | None = None, sh_degree: int = 0,
                  campos: Tensor | None = None, need_active: bool = True,
                  normalize_quats: bool = False, tile_mode: str = "radius") -> ViewsProjection:
    """gs3d/api.py:132-189 for every camera of a batch in one launch
    (splat_project_forward_views): bit-identical to one project_fused call
    per camera, with each Gaussian's inputs and SH row read once.
    views/projections (V,4,4), intrinsics (V,3,3), campos (V,3) or None."""
    pin = Args()
    V, n = views.shape[0], len(means)
    dev = means.device
    centers = [means.new_empty((n, 2)) for _ in range(V)]
    conics = [means.new_empty((n, 4)) for _ in range(V)]
    colors = [means.new_empty((n, 3)) for _ in range(V)] if sh is not None else None
    radii = torch.empty((V, n), dtype=torch.int32, device=dev)
    tiles = torch.empty((V, n), dtype=torch.int32, device=dev)
    depths = means.new_empty((V, n))
    active = (torch.empty((V, n, 3), dtype=torch.uint8, device=dev)
              if sh is not None and need_active else None)
    m2d, mop, mcon = means.new_empty((V, n, 2)), means.new_empty((V, n)), means.new_empty((V, n, 3))
    if n and V:
        sh_c = _c(sh)
        check(lib.splat_project_forward_views(
            V, n, pin(means), pin(quats), int(normalize_quats), pin(scales), pin(opacities),
            pin(views), pin(projections), pin(intrinsics), width, height, float(near), _far(far),
            float(radius_clip), pointer_table(centers), pointer_table(conics),
            pointer_table(radii), pointer_table(tiles), pointer_table(depths), int(sh_degree),
            sh_c.shape[1] if sh_c is not None else 0, ptr(sh_c), pin(campos),
            pointer_table(colors) if colors is not None else None, 3,
            pointer_table(active) if active is not None else None, pointer_table(m2d),
            pointer_table(mop), pointer_table(mcon), _tile_mode(tile_mode), _stream(means)),
            "project_forward_views")
    return ViewsProjection(centers, conics, colors, radii, tiles, depths, active, m2d, mop, mcon)


def metadata(state: ProjectedGaussians) -> dict[str, Tensor]:
    """splatting/metadata.py:34-70 prepare_metadata."""
    n = len(state.radii)
    means2d = torch.empty_like(state.centers)
    opacities = state.conics.new_empty((n,))
    conics = state.conics.new_empty((n, 3))
    if n:
        check(lib.splat_metadata(n, ptr(state.radii), ptr(state.centers), ptr(state.conics),
                                 ptr(means2d), ptr(opacities), ptr(conics),
                                 _stream(state.radii)), "metadata")
    return dict(radii=state.radii[:, None].expand(-1, 2), means2d=means2d, opacities=opacities,
                tiles_per_gauss=state.tile_counts, conics=conics)


def project_backward(means, quats, scales, opacities, view, projection, intrinsics, width,
                     height, state: ProjectedGaussians, grad_centers, grad_conics,
                     needs: tuple[bool, ...]):
    """gs3d/projection.py:357-428: [means, quats, scales, opacities, view, proj] grads."""
    pin = Args()
    if not any(needs):
        return [None] * 6
    tensors = [means, quats, scales, opacities]
    grads = [torch.empty_like(t) if need else None for t, need in zip(tensors, needs[:4])]
    n = len(means)
    cam = means.new_zeros(32) if any(needs[4:]) else None
    if n:
        check(lib.splat_project_backward(
            n, pin(means), pin(quats), pin(scales), pin(view),
            pin(projection), pin(intrinsics), width, height, ptr(state.radii),
            pin(grad_centers), pin(grad_conics), *[ptr(g) for g in grads], ptr(cam),
            _stream(means)), "project_backward")
    out = grads + [None, None]
    if needs[4]:
        out[4] = cam[:16].reshape(4, 4) if n else torch.zeros_like(view)
    if needs[5]:
        out[5] = cam[16:32].reshape(4, 4) if n else torch.zeros_like(projection)
    return out


# ---- spherical harmonics -----------------------------------------------------

def sh_forward(coeffs: Tensor, dirs: Tensor, degree: int, radii: Tensor | None, save: bool):
    pin = Args()
    n = len(coeffs)
    coeffs, dirs = coeffs.contiguous(), dirs.contiguous()
    colors = coeffs.new_empty((n, 3))
    active = torch.empty((n if save else 0, 3), dtype=torch.uint8, device=coeffs.device)
    if n:
        check(lib.splat_sh_forward(n, degree, coeffs.shape[1], ptr(coeffs), ptr(dirs),
                                   pin(radii), ptr(colors), ptr(active) if save else None,
                                   _stream(coeffs)), "sh_forward")
    return colors, active


def sh_backward(coeffs, dirs, degree, radii, active, upstream, need_dirs: bool):
    pin = Args()
    n = len(coeffs)
    coeffs, dirs = coeffs.contiguous(), dirs.contiguous()
    grad_coeffs = torch.empty_like(coeffs)
    grad_dirs = dirs.new_empty((n, 3)) if need_dirs else None
    if radii is None:
        radii_p = None
    else:
        radii_p = pin(radii)
    if n:
        check(lib.splat_sh_backward(n, degree, coeffs.shape[1], ptr(coeffs), ptr(dirs), radii_p,
                                    pin(active), pin(upstream),
                                    ptr(grad_coeffs), ptr(grad_dirs), _stream(coeffs)),
              "sh_backward")
    return grad_coeffs, grad_dirs


# ---- scan / binning ----------------------------------------------------------

def scan_counts(counts: Tensor) -> tuple[Tensor, int]:
    """primitives/tiling.py:57-64: inclusive int32 offsets and the total."""
    pin = Args()
    n = len(counts)
    offsets = torch.empty(n, dtype=torch.int32, device=counts.device)
    if not n:
        return offsets, 0
    ws = torch.empty(lib.splat_scan_workspace_bytes(n), dtype=torch.uint8, device=counts.device)
    total = torch.zeros(1, dtype=torch.int64, device=counts.device)
    check(lib.splat_scan_counts(n, pin(counts), ptr(offsets), ptr(total), ptr(ws),
                                ws.numel(), _stream(counts)), "scan_counts")
    value = int(total.item())
    if value > 2**31 - 1:
        nv.device_error(counts.device)  # clears the -4 this call recorded
        raise nv.SplatError(f"scan_counts: total {value} exceeds the int32 offsets")
    return offsets, value


# pair-count capacity of the last binning per (n, width, height, tile mode,
# view slot): lets the chunked emit run before the host has read the count
_PAIR_CAPACITY: dict[tuple, int] = {}


# the emission's pair limit (splat_bin_emit returns kTooLarge at 2^30 pairs)
_MAX_PAIR_CAPACITY = (1 << 30) - 1


def _capacity_for(pairs: int) -> int:
    """The early emission's id capacity for the next call: the last count
    plus 12.5 %, clamped to the emission limit (a count above it is emitted
    again exactly after the host read)."""
    return min(pairs + pairs // 8 + 4096, _MAX_PAIR_CAPACITY)


class BinPlan:
    """Phase 1 of binning for one view (depth sort, offsets, ranges, count)."""

    def __init__(self, state: ProjectedGaussians, width: int, height: int,
                 tile_mode: str = "radius"):
        dev = state.radii.device
        n = len(state.radii)
        self.mode = _tile_mode(tile_mode)
        self.n, self.width, self.height = n, width, height
        self.state = state
        gx, gy = (width + 15) // 16, (height + 15) // 16
        self.ranges = torch.empty((gx * gy, 2), dtype=torch.int32, device=dev)
        # written by splat_bin_prepare (the total, or 0 without Gaussians)
        self.pairs_dev = torch.empty(1, dtype=torch.int64, device=dev)
        self.workspace = torch.empty(lib.splat_bin_workspace_bytes(n, width, height, self.mode),
                                     dtype=torch.uint8, device=dev)
        self.pin = Args()  # the projected rows stay referenced until emit
        # the chunked scatter needs no pair workspace and accepts a capacity
        self.chunked = lib.splat_bin_pairs_workspace_bytes(1, width, height, self.mode) == 0
        self.early: Tensor | None = None
        pin = self.pin
        check(lib.splat_bin_prepare(
            n, pin(state.centers), pin(state.conics), pin(state.radii), pin(state.tile_counts),
            pin(state.depths), width, height, self.mode, ptr(self.workspace),
            self.workspace.numel(), ptr(self.ranges), ptr(self.pairs_dev), nv.stream(dev)),
            "bin_prepare")

    def emit_early(self, capacity: int) -> None:
        """Queue the chunked emit into a capacity-sized buffer before the
        pair count is known on the host (finish() checks it)."""
        dev = self.ranges.device
        self.early = torch.empty(capacity, dtype=torch.int32, device=dev)
        pin, st = self.pin, self.state
        check(lib.splat_bin_emit(self.n, capacity, self.width, self.height, self.mode,
                                 pin(st.centers), pin(st.conics), pin(st.radii),
                                 ptr(self.workspace), self.workspace.numel(), None, 0,
                                 ptr(self.early), nv.stream(dev)), "bin_emit")

    def finish(self, pairs: int) -> Tensor:
        """point_list of `pairs` entries: the early emit's when it fitted,
        else an exact emit now."""
        if self.early is not None and pairs <= len(self.early):
            ids = self.early[:pairs]
            self.early = self.workspace = self.pin = None
            return ids
        self.early = None
        return self.emit(pairs)

    def emit(self, pairs: int) -> Tensor:
        dev = self.ranges.device
        ids = torch.empty(pairs, dtype=torch.int32, device=dev)
        if pairs:
            pws = torch.empty(lib.splat_bin_pairs_workspace_bytes(pairs, self.width, self.height,
                                                                  self.mode),
                              dtype=torch.uint8, device=dev)
            pin, st = self.pin, self.state
            check(lib.splat_bin_emit(self.n, pairs, self.width, self.height, self.mode,
                                     pin(st.centers), pin(st.conics), pin(st.radii),
                                     ptr(self.workspace), self.workspace.numel(), ptr(pws),
                                     pws.numel(), ptr(ids), nv.stream(dev)), "bin_emit")
        self.workspace = None
        self.pin = None
        return ids


_DEVICE_ERRORS = {-3: "a bounded device wait expired (look-back timeout)",
                  -4: "a count total exceeded INT32_MAX",
                  -6: "a device guard met an out-of-range index (inconsistent input)"}


def raise_device_error(code: int) -> None:
    """Raise SplatError for a non-zero device error word: the binning of this
    call (or the kernels queued since the last read) cannot be trusted."""
    if code:
        raise nv.SplatError(f"device error {code}: {_DEVICE_ERRORS.get(code, 'unknown code')}")


def bin_and_sort_many(states: list[ProjectedGaussians], width: int, height: int,
                      camera_status: list | None = None, tile_mode: str = "radius",
                      host_reads: list[Tensor] | None = None):
    """Bin several views with one host read of all pair counts.

    camera_status: deferred camera status tensors (cameras_prepare's
    status_sink); they are read in the same synchronisation and their errors
    raised before any pair is emitted.  host_reads: further integer scalars
    the caller needs on the host, read in that same synchronisation; when
    given, (bins, their values) is returned."""
    plans = [BinPlan(s, width, height, tile_mode) for s in states]
    # the blend schedule needs only the ranges: queued before the host read,
    # so nothing but the emits waits for the pair counts
    orders = [tile_order(dict(ranges=p.ranges)) for p in plans]
    parts = [p.pairs_dev for p in plans]
    ncodes = 0
    if camera_status:
        codes_dev = torch.cat([c.to(torch.int64) for c in camera_status])
        ncodes = len(codes_dev)
        parts = [codes_dev] + parts
    extra = [t.reshape(1).to(torch.int64) for t in (host_reads or [])]
    parts = parts + extra
    # the device error word (bounded waits that expired, guards that met an
    # out-of-range index) rides along in the same read and is reset behind it
    err_word = None
    if plans:
        err_word = torch.empty(1, dtype=torch.int32, device=plans[0].ranges.device)
        check(lib.splat_device_error_read(ptr(err_word), nv.stream(err_word.device)),
              "device_error_read")
        parts = parts + [err_word.to(torch.int64)]
    values: list = []
    keys = [(p.n, width, height, p.mode, v) for v, p in enumerate(plans)]
    if parts:
        # the counts travel to pinned memory behind an event; chunked emits
        # with a capacity from the last call are queued after that copy, so
        # the GPU scatters while the host waits for (only) the counts
        dev_values = torch.cat(parts)
        host = torch.empty(len(dev_values), dtype=torch.int64, pin_memory=True)
        host.copy_(dev_values, non_blocking=True)
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(dev_values.device))
        for key, p in zip(keys, plans):
            capacity = _PAIR_CAPACITY.get(key)
            if p.chunked and capacity:
                p.emit_early(capacity)
        ready.synchronize()
        values = host.tolist()
    if err_word is not None:
        raise_device_error(int(values.pop()))
    raise_camera_errors(values[:ncodes])
    counts = values[ncodes:ncodes + len(plans)]
    bins = []
    for key, p, m, o in zip(keys, plans, counts, orders):
        bins.append(dict(point_list=p.finish(int(m)), ranges=p.ranges, tile_order=o))
        if p.chunked:
            _PAIR_CAPACITY[key] = _capacity_for(int(m))
    if host_reads is None:
        return bins
    return bins, values[ncodes + len(plans):]


def bin_and_sort(state: ProjectedGaussians, width: int, height: int,
                 tile_mode: str = "radius") -> dict[str, Tensor]:
    """splatting/binning.py:72-117: point_list and ranges.  state.tile_counts
    must come from the projection with the same tile_mode."""
    return bin_and_sort_many([state], width, height, tile_mode=tile_mode)[0]


# ---- blending ----------------------------------------------------------------

def tile_order(bins: dict) -> Tensor:
    """The blend's block schedule for these bins: tiles by descending pair
    count (splat_tile_order), computed once per bins dict and cached in it."""
    order = bins.get("tile_order")
    if order is None:
        ranges = bins["ranges"]
        order = torch.empty(len(ranges), dtype=torch.int32, device=ranges.device)
        check(lib.splat_tile_order(ptr(ranges), len(ranges), ptr(order),
                                   nv.stream(ranges.device)), "tile_order")
        bins["tile_order"] = order
    return order


def _features(feat_a: Tensor, feat_b: Tensor | None):
    a = feat_a.contiguous()
    b = None if feat_b is None else feat_b.contiguous()
    return a, b, a.shape[1], (0 if b is None else b.shape[1])


def render(state: ProjectedFootprint, bins: dict, feat_a: Tensor, feat_b: Tensor | None,
           append_one: bool, background: Tensor, width: int, height: int,
           planar: bool = False, statistics=None, separate_alpha: bool = False) -> RenderedPixels:
    """gs3d/render.py:359-406.  Channels: feat_a, feat_b, then a constant 1.

    statistics: a PreparedStatistics (statistics.py) whose counts/sums rows
    receive this view's accepted contributions.  separate_alpha (interleaved,
    append_one): the constant channel -- alpha -- goes to its own (H, W, 1)
    buffer and features hold the other channels."""
    pin = Args()
    a, b, ca, cb = _features(feat_a, feat_b)
    channels = ca + cb + int(append_one)
    dev = a.device
    if separate_alpha and (planar or not append_one):
        raise ValueError("separate_alpha needs interleaved output with the constant channel")
    alpha = a.new_empty((height, width, 1)) if separate_alpha else None
    stored = channels - int(separate_alpha)
    if planar:
        image = a.new_empty((channels, height, width))
        pix_stride, ch_stride = 1, height * width
    else:
        image = a.new_empty((height, width, stored))
        pix_stride, ch_stride = stored, 1
    out = RenderedPixels(image, a.new_empty((height, width)),
                         torch.empty((height, width), dtype=torch.int32, device=dev), alpha)
    if statistics is None:
        stat = (0, 0, None, None, None)
    else:
        mask = sum(1 << r for r, kind in enumerate(statistics.key) if kind == 1)
        stat = (len(statistics.key), mask, ptr(statistics.pixel_values),
                ptr(statistics.counts), ptr(statistics.sums))
    with _timed("render_forward", dev):
        check(lib.splat_render_forward_statistics(
            width, height, ptr(bins["ranges"]), ptr(bins["point_list"]), len(bins["point_list"]),
            len(state.centers), pin(state.centers),
            pin(state.conics), ptr(a), ca, ca, ptr(b), cb, cb, int(append_one),
            pin(background), ptr(image), pix_stride, ch_stride, ptr(alpha),
            ptr(out.transmittance), ptr(out.contributors), *stat, ptr(tile_order(bins)),
            nv.stream(dev)), "render_forward")
    return out


def render_backward(state: ProjectedFootprint, bins: dict, feat_a: Tensor,
                    feat_b: Tensor | None, append_one: bool, background: Tensor,
                    final_t: Tensor, contributors: Tensor, gradient: Tensor | None, width: int,
                    height: int, *, planar: bool = False, absgrad: bool = False,
                    constant_tail: int = 0, need_a: bool = True, need_b: bool = True,
                    gradient_alpha: Tensor | None = None, separate_alpha: bool = False,
                    absolute_out: Tensor | None = None, centers_out: Tensor | None = None,
                    separate_buffers: bool = False):
    """gs3d/render.py:409-463: grads of centers, conics, feat_a, feat_b, abs.

    separate_alpha: gradient holds the channels before the constant one
    (H, W, C'-1) and gradient_alpha (H, W, 1) the constant channel's; either
    may be None (zero).  absolute_out: a zeroed contiguous (n, 2) buffer that
    receives the |d centers| sums in place of a new one; centers_out: a zeroed
    contiguous (n, 2) buffer that receives the centre gradient likewise.
    separate_buffers: the conic and feature gradients get allocations of
    their own (outputs of a Torch custom op must not alias one another);
    otherwise they are views of one zero fill."""
    pin = Args()
    a, b, ca, cb = _features(feat_a, feat_b)
    channels = ca + cb + int(append_one)
    if not 0 <= constant_tail <= channels:
        raise ValueError("constant_tail must be within the feature channel count")
    if separate_alpha and (planar or not append_one):
        raise ValueError("separate_alpha needs interleaved output with the constant channel")
    stored = channels - int(separate_alpha)
    g = None if gradient is None else gradient.contiguous()
    g_alpha = None if gradient_alpha is None else gradient_alpha.contiguous()
    alpha_stride = 1
    if separate_alpha and g_alpha is None:
        # the constant channel's upstream is not in `gradient`: read zero
        g_alpha, alpha_stride = a.new_zeros(1), 0
    if planar:
        pix_stride, ch_stride = 1, height * width
    else:
        pix_stride, ch_stride = stored, 1
    centers = centers_out if centers_out is not None else torch.zeros_like(state.centers)
    # the conic and first feature gradients share one zero fill (conics first:
    # their rows stay 16-byte aligned)
    if separate_buffers:
        conics = torch.zeros_like(state.conics)
        ga = torch.zeros_like(a) if need_a else None
    else:
        n_rows = len(state.conics)
        flat = state.conics.new_zeros(n_rows * 4 + (a.numel() if need_a else 0))
        conics = flat[:n_rows * 4].view(state.conics.shape)
        ga = flat[n_rows * 4:].view(a.shape) if need_a else None
    gb = torch.zeros_like(b) if (b is not None and need_b) else None
    if absgrad:
        absolute = absolute_out if absolute_out is not None else torch.zeros_like(state.centers)
    else:
        absolute = None
    with _timed("render_backward", a.device):
        check(lib.splat_render_backward(
            width, height, ptr(bins["ranges"]), ptr(bins["point_list"]), len(bins["point_list"]),
            len(state.centers), pin(state.centers),
            pin(state.conics), ptr(a), ca, ca, ptr(b), cb, cb, int(append_one),
            pin(background), pin(final_t), pin(contributors),
            ptr(g), pix_stride, ch_stride, ptr(g_alpha), alpha_stride, ptr(centers), ptr(conics), ptr(ga),
            ptr(gb), ptr(absolute), constant_tail, ptr(tile_order(bins)), nv.stream(a.device)),
            "render_backward")
    return centers, conics, ga, gb, absolute
