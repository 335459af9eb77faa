"""AAA-Gaussians stage wrappers over the C ABI (include/splat200.h).

The L2 swap points of dsl_splat/aaa for one view, each allocating its
outputs with Torch (as the reference's wrappers do) and enqueuing the
sm_100a kernels on the current stream:

  preprocess        aaa/preprocess.py:165-560 (eval_3D: preprocess_3d, then
                    cull_remainder_3d when load-balanced)
  bin_and_sort_many aaa/binning.py:278-342 (one host read of every view's
                    pair count, as the reference's single .item())
  render            aaa/render_hierarchical_warp.py:694-801
  render_backward   aaa/backward_render.py:140-248
  preprocess_backward aaa/backward_preprocess.py:270-346
  camera_backward   aaa/backward_camera.py:225-294
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import Tensor

from .. import _native as nv
from .. import stages as core
from .._native import check, lib, ptr
from .settings import ExtendedSettings

Args = core.Args


@dataclass(slots=True)
class AaaView:
    """One lowered camera (the FrameConfig fields the kernels read)."""

    width: int
    height: int
    tanfovx: float
    tanfovy: float
    principal: tuple[float, float]
    viewmatrix: Tensor   # (4,4) V^T storage
    projmatrix: Tensor   # (4,4) (P V)^T storage
    campos: Tensor       # (3)
    scale_modifier: float = 1.0


@dataclass(slots=True)
class AaaState:
    """PreprocessedGaussians (aaa/types.py:31-54) of the eval_3D path: only
    rows with radii > 0 define geometry."""

    centers: Tensor      # means2D (N,2): bounding centre
    rects: Tensor        # rects2D (N,2): bounding half extents
    depths: Tensor
    transforms: Tensor   # gauss2screen (N,4,4)
    opacity: Tensor      # effective opacity (N)
    radii: Tensor
    tiles: Tensor        # tiles_touched
    valid: Tensor        # bool (N)
    # the quaternions given to the kernels are raw: they normalise them (with
    # F.normalize's bits) and the preprocessing adjoint returns their gradient
    raw_quats: bool = False


def default_binning(settings: ExtendedSettings) -> bool:
    """aaa/binning.py:205-213: the load-balanced key emission these kernels
    implement (the other combinations use the reference's generic emission,
    which is not built here)."""
    return (bool(settings.eval_3D) and bool(settings.load_balancing)
            and bool(settings.culling_settings.tile_based_culling)
            and int(settings.sort_settings.sort_order) == 3)


def require_supported(settings: ExtendedSettings) -> None:
    if not default_binning(settings):
        raise NotImplementedError(
            "the B200 AAA path implements the load-balanced binning (eval_3D, "
            "load_balancing, tile_based_culling, sort_order PTD_MAX)")


def frame(view: AaaView, settings: ExtendedSettings, means: Tensor, quats: Tensor,
          scales: Tensor, opacities: Tensor, filters: Tensor | None, pin: Args,
          sh: Tensor | None = None, sh_degree: int = 0, flags: dict | None = None,
          raw_quats: bool = False):
    """The SplatAaaFrame of one view (device pointers kept alive by pin).

    flags overrides the preprocessing switches (the golden tests drive
    preprocess_3d with the reference's raw flags); by default they follow
    aaa/preprocess.py:202-323 from the settings."""
    f = nv.SplatAaaFrame()
    n = len(means)
    f.n, f.width, f.height = n, view.width, view.height
    f.means, f.scales, f.quats, f.opacities = (pin(means), pin(scales), pin(quats),
                                               pin(opacities.reshape(n)))
    f.sh = pin(sh) if sh is not None else None
    f.sh_k = sh.shape[1] if sh is not None else 0
    f.sh_degree = sh_degree
    f.filters = pin(filters.reshape(n)) if filters is not None else None
    f.campos, f.view, f.proj = pin(view.campos.reshape(3)), pin(view.viewmatrix), pin(view.projmatrix)
    f.tanfov_x, f.tanfov_y = view.tanfovx, view.tanfovy
    f.principal_x, f.principal_y = view.principal
    f.scale_modifier = view.scale_modifier
    # the adjoints' focal lengths, in double as the reference's host computes them
    f.focal_x = view.width / (2.0 * view.tanfovx)
    f.focal_max = max(view.width / (2 * view.tanfovx), view.height / (2 * view.tanfovy))
    culling = settings.culling_settings
    cooperative = bool(settings.load_balancing and culling.tile_based_culling)
    values = dict(sort_order=int(settings.sort_settings.sort_order),
                  ewa=bool(settings.proper_ewa_scaling),
                  new_aabb=bool(getattr(settings, "new_aabb", True)),
                  near_clipping=bool(getattr(settings, "near_clipping", False)),
                  tile_culling=bool(culling.tile_based_culling),
                  complete=bool(settings.eval_3D) and not cooperative, cooperative=cooperative,
                  normalize_quats=raw_quats)
    values.update(flags or {})
    for name, value in values.items():
        setattr(f, name, int(value))
    return f


def preprocess(view: AaaView, settings: ExtendedSettings, means: Tensor, quats: Tensor,
               scales: Tensor, opacities: Tensor, filters: Tensor | None = None,
               radius_clip: float = 0.0, raw_quats: bool = False) -> AaaState:
    """aaa/preprocess.py:165-560 + aaa/frame.py:51-58 (radius clip); raw_quats:
    quats are unnormalised (the kernels normalise them)."""
    n, dev = len(means), means.device
    pin = Args()
    f = frame(view, settings, means, quats, scales, opacities, filters, pin, raw_quats=raw_quats)
    empty = lambda *shape: torch.empty(shape, device=dev, dtype=torch.float32)  # noqa: E731
    st = AaaState(empty(n, 2), empty(n, 2), empty(n), empty(n, 4, 4), empty(n),
                  torch.empty(n, device=dev, dtype=torch.int32),
                  torch.empty(n, device=dev, dtype=torch.int32),
                  torch.empty(n, device=dev, dtype=torch.uint8), raw_quats)
    queued = torch.empty(max(n, 1), device=dev, dtype=torch.int32)
    size = torch.empty(1, device=dev, dtype=torch.int32)
    s = nv.stream(dev)
    check(lib.splat_aaa_preprocess(
        ctypes_ref(f), ptr(st.centers), ptr(st.rects), ptr(st.depths), ptr(st.transforms),
        ptr(st.opacity), ptr(st.radii), ptr(st.tiles), None, ptr(st.valid), None, ptr(queued),
        ptr(size), s), "aaa_preprocess")
    if f.cooperative:
        check(lib.splat_aaa_cull_remainder(
            n, ptr(queued), ptr(size), ptr(st.centers), ptr(st.rects), ptr(st.transforms),
            ptr(st.opacity), view.width, view.height, ptr(st.radii), ptr(st.tiles),
            ptr(st.valid), s), "aaa_cull_remainder")
    st.valid = st.valid.view(torch.bool)
    if radius_clip > 0:
        keep = st.radii > radius_clip
        st.radii = torch.where(keep, st.radii, 0)
        st.tiles = torch.where(keep, st.tiles, 0)
        st.valid = st.valid & keep
    return st


def ctypes_ref(f) -> int:
    """Host address of a SplatAaaFrame for the call (kept alive by the caller)."""
    import ctypes
    return ctypes.addressof(f)


def bin_and_sort_many(states: list[AaaState], width: int, height: int,
                      host_reads: list[Tensor] | None = None):
    """aaa/binning.py:278-342 for several views: the tile-count scans, one
    host read of every pair count (and of host_reads, the caller's scalars,
    with the device error word), then per view the emission, sort and
    ranges.  Returns the bins (point_list, ranges, tile_order) and the
    host_reads values."""
    dev = states[0].radii.device if states else torch.device("cuda")
    gx, gy = (width + 15) // 16, (height + 15) // 16
    scans = []
    for st in states:
        n = len(st.radii)
        offsets = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
        total = torch.zeros(1, dtype=torch.int64, device=dev)
        if n:
            ws = torch.empty(lib.splat_scan_workspace_bytes(n), dtype=torch.uint8, device=dev)
            check(lib.splat_scan_counts(n, ptr(st.tiles), ptr(offsets), ptr(total), ptr(ws),
                                        ws.numel(), nv.stream(dev)), "aaa scan_counts")
        scans.append((offsets, total))
    err = torch.empty(1, dtype=torch.int32, device=dev)
    check(lib.splat_device_error_read(ptr(err), nv.stream(dev)), "device_error_read")
    parts = [t for _, t in scans] + [t.reshape(1).to(torch.int64) for t in (host_reads or [])]
    parts.append(err.to(torch.int64))
    values = torch.cat(parts).tolist()  # the host synchronisation
    core.raise_device_error(int(values.pop()))
    bins = []
    for st, (offsets, _), m in zip(states, scans, values):
        m = int(m)
        if m > 2**31 - 1:
            raise nv.SplatError(f"aaa binning: {m} pairs exceed the int32 offsets")
        ranges = torch.empty((gx * gy, 2), dtype=torch.int32, device=dev)
        ids = torch.empty(m, dtype=torch.int32, device=dev)
        ws = torch.empty(lib.splat_aaa_bin_workspace_bytes(m), dtype=torch.uint8, device=dev)
        check(lib.splat_aaa_bin(len(st.radii), m, ptr(offsets), ptr(st.centers), ptr(st.rects),
                                ptr(st.radii), ptr(st.transforms), ptr(st.opacity), width, height,
                                ptr(ws), ws.numel(), ptr(ids), ptr(ranges), nv.stream(dev)),
              "aaa_bin")
        b = dict(point_list=ids, ranges=ranges)
        b["tile_order"] = core.tile_order(b)
        bins.append(b)
    return bins, values[len(states):]


def metadata(view_matrix: Tensor, focal: tuple[float, float], principal: tuple[float, float],
             means: Tensor, state: AaaState, radii: Tensor, means2d: Tensor,
             opacities: Tensor) -> None:
    """aaa/metadata.py:55-91 _geometry of one view into preallocated rows:
    radii (N,2) int32 = ceil of the half extents, means2d (N,2) the pixel
    projection of the means, opacities (N) the effective opacities; zeros
    where state.radii <= 0.  view_matrix: (4,4) world-to-camera."""
    n = len(means)
    if n == 0:
        return
    pin = Args()
    check(lib.splat_aaa_metadata(n, pin(view_matrix.contiguous()), float(focal[0]),
                                 float(focal[1]), float(principal[0]), float(principal[1]),
                                 pin(means), ptr(state.rects), ptr(state.radii),
                                 ptr(state.opacity), ptr(radii), ptr(means2d), ptr(opacities),
                                 nv.stream(means.device)), "aaa_metadata")


# Blend records kept by the forward for the backward: per pixel up to this
# many blended samples (at most 256; 8 bytes each; T*256*capacity slots,
# 3.2 GB at 1080p, of which only the blended samples are written and read);
# a pixel past it sends its tile to the replay kernel.  The 2M-Gaussian
# 1080p benchmark scene (bench.py --config 3) blends 63 samples per pixel on
# average, at most 146.  The backward consumes the records (it overwrites
# them); a second backward of the same forward replays.
RECORD_CAPACITY = 192


def render(state: AaaState, bins: dict, features: Tensor, background: Tensor, width: int,
           height: int, cull: bool, record_capacity: int = 0, statistics=None):
    """aaa/render_hierarchical_warp.py:694-801: color (C,H,W), final_T and
    contributors (H,W); with record_capacity > 0 also the blend records
    (a dict the backward takes), else None.  statistics: a
    PreparedStatistics whose counts / sums receive the view's contribution
    statistics (render_statistics, :608-653)."""
    dev = features.device
    C = features.shape[1]
    image = torch.empty((C, height, width), device=dev, dtype=torch.float32)
    final_t = torch.empty((height, width), device=dev, dtype=torch.float32)
    contrib = torch.empty((height, width), device=dev, dtype=torch.int32)
    if features.shape[0] == 0:  # nothing blends: colour 0, transmittance 1
        image.zero_()
        final_t.fill_(1.0)
        contrib.zero_()
        return image, final_t, contrib, None
    records = None
    if record_capacity > 0:
        tiles = ((width + 15) // 16) * ((height + 15) // 16)
        slots = tiles * 256 * record_capacity
        records = dict(capacity=record_capacity,
                       entries=torch.empty((slots, 2), device=dev, dtype=torch.float32),
                       counts=torch.empty(tiles * 256, device=dev, dtype=torch.int32),
                       overflow=torch.empty(tiles, device=dev, dtype=torch.int32))
    rec = records or {}
    pin = Args()
    stats = statistics
    stat_count = len(stats.key) if stats is not None else 0
    stat_mask = sum(1 << r for r, k in enumerate(stats.key) if k == 1) if stat_count else 0
    with core._timed("aaa_render_forward", dev):
        check(lib.splat_aaa_render(features.shape[0], width, height, C, int(cull),
                                   ptr(bins["ranges"]), ptr(bins["point_list"]),
                                   pin(state.transforms), pin(state.opacity), pin(features),
                                   pin(background), ptr(bins.get("tile_order")), ptr(image),
                                   ptr(final_t), ptr(contrib), rec.get("capacity", 0),
                                   ptr(rec.get("entries")), ptr(rec.get("counts")),
                                   ptr(rec.get("overflow")), stat_count, stat_mask,
                                   pin(stats.pixel_values) if stat_count else None,
                                   ptr(stats.counts) if stat_count else None,
                                   ptr(stats.sums) if stat_count else None,
                                   nv.stream(dev)), "aaa_render")
    return image, final_t, contrib, records


def render_backward(state: AaaState, bins: dict, features: Tensor, background: Tensor,
                    image: Tensor, final_t: Tensor, grad_image: Tensor, width: int, height: int,
                    cull: bool, screen: bool = False, absgrad: bool = False,
                    records: dict | None = None):
    """aaa/backward_render.py:140-248: gradients of the transforms (N,4,4,
    the reference's transposed layout), effective opacities (N), features
    (N,C) and, when asked, the screen translations (N,2) and their absolute
    per-pixel sums (N,2) -- disjoint views of one zero-filled buffer."""
    if absgrad and not screen:
        raise ValueError("absgrad requires screen_grad=True")
    n, C = features.shape
    dev = features.device
    screen_channels = 2 * (int(screen) + int(absgrad))
    storage = torch.zeros(n * (17 + C + screen_channels), device=dev, dtype=torch.float32)
    g_tr = storage[: 16 * n].view(n, 4, 4)
    g_col = storage[16 * n: (16 + C) * n].view(n, C)
    g_op = storage[(16 + C) * n: (17 + C) * n]
    g_scr = storage[(17 + C) * n: (19 + C) * n].view(n, 2) if screen else None
    g_abs = storage[(19 + C) * n: (21 + C) * n].view(n, 2) if absgrad else None
    if records is not None and records.get("consumed"):
        records = None  # a second backward of the same forward replays the queues
    if n:
        pin = Args()
        rec = records or {}
        with core._timed("aaa_render_backward", dev):
            check(lib.splat_aaa_render_backward(
                n, width, height, C, int(cull), ptr(bins["ranges"]), ptr(bins["point_list"]),
                pin(state.transforms), pin(state.opacity), pin(features), pin(background),
                ptr(bins.get("tile_order")), pin(image), pin(final_t), pin(grad_image), ptr(g_tr),
                ptr(g_op), ptr(g_col), ptr(g_scr), ptr(g_abs), rec.get("capacity", 0),
                ptr(rec.get("entries")), ptr(rec.get("counts")), ptr(rec.get("overflow")),
                nv.stream(dev)), "aaa_render_backward")
        if records is not None:
            records["consumed"] = True  # the backward overwrote the entries
    return g_tr, g_op, g_col, g_scr, g_abs


def preprocess_backward(view: AaaView, settings: ExtendedSettings, means: Tensor, quats: Tensor,
                        scales: Tensor, opacities: Tensor, state: AaaState, grad_transforms: Tensor,
                        grad_opacity: Tensor):
    """aaa/backward_preprocess.py:270-346: (opacities, means, scales, quats)
    gradients (of the raw quaternions when state.raw_quats)."""
    n, dev = len(means), means.device
    g_o = torch.empty(n, device=dev)
    g_m = torch.empty((n, 3), device=dev)
    g_s = torch.empty((n, 3), device=dev)
    g_q = torch.empty((n, 4), device=dev)
    if n:
        pin = Args()
        f = frame(view, settings, means, quats, scales, opacities, None, pin,
                  raw_quats=state.raw_quats)
        check(lib.splat_aaa_preprocess_backward(
            ctypes_ref(f), ptr(state.radii), pin(grad_transforms), pin(grad_opacity), ptr(g_o),
            ptr(g_m), ptr(g_s), ptr(g_q), nv.stream(dev)), "aaa_preprocess_backward")
    return g_o, g_m, g_s, g_q


def camera_backward(view: AaaView, settings: ExtendedSettings, means: Tensor, quats: Tensor,
                    scales: Tensor, filters: Tensor | None, state: AaaState,
                    grad_transforms: Tensor, grad_opacity: Tensor):
    """aaa/backward_camera.py:225-294: gradients of the viewmatrix, projmatrix
    and campos tensors (the lowered camera's storage)."""
    dev = means.device
    sums = torch.empty(23, device=dev)
    pin = Args()
    f = frame(view, settings, means, quats, scales, state.opacity, filters, pin,
              raw_quats=state.raw_quats)
    check(lib.splat_aaa_camera_backward(ctypes_ref(f), ptr(state.radii), pin(state.opacity),
                                        pin(grad_transforms), pin(grad_opacity), ptr(sums),
                                        nv.stream(dev)), "aaa_camera_backward")
    g_view = torch.zeros((4, 4), device=dev)
    g_view[:, 2] = sums[16:20]
    return g_view, sums[:16].view(4, 4), sums[20:23]


__all__ = ["AaaView", "AaaState", "RECORD_CAPACITY", "preprocess", "metadata", "bin_and_sort_many",
           "render", "render_backward", "preprocess_backward", "camera_backward",
           "default_binning"]
