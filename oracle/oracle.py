"""ctypes bindings for the CPU oracle (test infrastructure only).

The oracle restates dsl_splat's gs3d rasteriser, its RaDe-GS projection
and render, and the AAA-Gaussians preprocessing on the CPU (see
splat_oracle.cpp and aaa_oracle.cpp for the per-function reference
citations).  Tests,
``__graft_entry__.smoke()`` and bench.py's CPU legs use it as the checker and
the CPU baseline; the product package never imports it.

Every function takes and returns numpy arrays (float32 / int32, C order).
Gradient accumulators come back as float64.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libsplat_oracle.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(dtype=np.uint64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_vp = ctypes.c_void_p
_int = ctypes.c_int
_flt = ctypes.c_float


def build() -> None:
    """Compile the oracle library in place (make, with FP contraction off)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oracle_expf.argtypes = [_flt]
        L.oracle_expf.restype = _flt
        L.oracle_logf.argtypes = [_flt]
        L.oracle_logf.restype = _flt
        L.oracle_atan2f.argtypes = [_flt, _flt]
        L.oracle_atan2f.restype = _flt
        L.oracle_tanf.argtypes = [_flt]
        L.oracle_tanf.restype = _flt
        L.oracle_cameras_prepare.argtypes = [_int, _f32p, _f32p, _int, _int, _int, _vp, _vp, _vp, _i32p]
        L.oracle_cameras_prepare.restype = _int
        L.oracle_cameras_backward.argtypes = [_int, _f32p, _vp, _int, _int, _vp, _vp, _f32p]
        L.oracle_cameras_backward.restype = None
        L.oracle_project_forward.argtypes = [
            _int, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _int, _int,
            _flt, _flt, _flt, _f32p, _f32p, _i32p, _i32p, _f32p, _int]
        L.oracle_project_forward.restype = None
        L.oracle_sh_forward.argtypes = [_int, _int, _int, _f32p, _f32p, _vp, _f32p, _vp]
        L.oracle_sh_forward.restype = None
        L.oracle_sh_backward.argtypes = [_int, _int, _int, _f32p, _f32p, _vp, _u8p, _f32p, _f32p, _vp]
        L.oracle_sh_backward.restype = None
        L.oracle_scan_counts.argtypes = [_int, _i32p, _i32p]
        L.oracle_scan_counts.restype = ctypes.c_longlong
        L.oracle_bin_and_sort.argtypes = [_int, _f32p, _i32p, _f32p, _i32p, _int, _int, _u64p, _i32p, _i32p,
                                          _vp, _int]
        L.oracle_bin_and_sort.restype = None
        L.oracle_render_forward.argtypes = [
            _int, _int, _int, _i32p, _i32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _i32p]
        L.oracle_render_forward.restype = None
        L.oracle_render_backward.argtypes = [
            _int, _int, _int, _int, _i32p, _i32p, _f32p, _f32p, _f32p, _f32p, _f32p, _i32p,
            _f32p, _f64p, _f64p, _f64p, _vp]
        L.oracle_render_backward.restype = None
        L.oracle_project_backward.argtypes = [
            _int, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _int, _int, _i32p, _f32p,
            _f32p, _f32p, _f32p, _f32p, _f32p, _vp, _vp]
        L.oracle_project_backward.restype = None
        L.oracle_rade_project.argtypes = [
            _int, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _int, _int, _flt, _flt, _flt,
            _flt, _f32p, _f32p, _i32p, _i32p, _f32p, _f32p, _f32p]
        L.oracle_rade_project.restype = None
        L.oracle_rade_render.argtypes = [
            _int, _int, _int, _i32p, _i32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
            _f32p, _f32p, _i32p]
        L.oracle_rade_render.restype = None
        L.oracle_rade_render_backward.argtypes = [
            _int, _int, _int, _i32p, _i32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
            _f32p, _f32p, _i32p, _vp, _vp, _vp, _vp, _vp, _f64p, _f64p, _f64p, _vp, _f64p, _f64p]
        L.oracle_rade_render_backward.restype = None
        L.oracle_aaa_preprocess.argtypes = [
            _int, _f32p, _f32p, _f32p, _f32p, _vp, _int, _int, _int, _int, _vp, _f32p, _f32p,
            _f32p, _int, _int, _flt, _flt, _flt, _flt, _flt, _int, _int, _int, _int, _int, _int,
            _f32p, _f32p, _f32p, _f32p, _f32p, _i32p, _i32p, _vp, _u8p, _vp, _i32p, _i32p]
        L.oracle_aaa_preprocess.restype = None
        L.oracle_aaa_cull_remainder.argtypes = [
            _i32p, _int, _f32p, _f32p, _f32p, _f32p, _int, _int, _i32p, _i32p, _u8p]
        L.oracle_aaa_cull_remainder.restype = None
        L.oracle_aaa_duplicate.argtypes = [
            _int, _f32p, _f32p, _i32p, _f32p, _f32p, _i32p, _int, _int, _u64p, _i32p, _int]
        L.oracle_aaa_duplicate.restype = None
        L.oracle_aaa_preprocess_backward.argtypes = [
            _int, _f32p, _f32p, _f32p, _f32p, _i32p, _f32p, _f32p, _f32p, _int, _int, _flt, _int,
            _f32p, _f32p, _f32p, _f32p, _f32p, _f32p]
        L.oracle_aaa_preprocess_backward.restype = None
        L.oracle_aaa_camera_backward.argtypes = [
            _int, _f32p, _f32p, _f32p, _vp, _i32p, _f32p, _f32p, _f32p, _f32p, _int, _int, _flt,
            _flt, _int, _f32p, _f32p, _vp, _int, _int, _vp, _f32p, _f32p]
        L.oracle_aaa_camera_backward.restype = None
        L.oracle_aaa_render.argtypes = [
            _int, _int, _int, _i32p, _i32p, _f32p, _f32p, _f32p, _f32p, _int, _f32p, _f32p,
            _i32p, _int, _int, _int, _f32p, _i32p, _f64p]
        L.oracle_aaa_render.restype = _int
        L.oracle_aaa_render_backward.argtypes = [
            _int, _int, _int, _i32p, _i32p, _f32p, _f32p, _f32p, _f32p, _int, _f32p, _f32p,
            _f32p, _f64p, _f64p, _f64p, _vp, _vp]
        L.oracle_aaa_render_backward.restype = _int
        L.oracle_num_threads.restype = _int
        L.oracle_set_num_threads.argtypes = [_int]
        _lib = L
    return _lib


def _c(a, dtype=np.float32):
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def set_threads(n: int) -> None:
    lib().oracle_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def expf(x: np.ndarray) -> np.ndarray:
    f = lib().oracle_expf
    x = _c(x).ravel()
    return np.array([f(float(v)) for v in x], dtype=np.float32)


def atan2f(y: np.ndarray, x: np.ndarray) -> np.ndarray:
    """aaa_oracle.cpp oracle_atan2f element-wise (the AAA bounds' atan2)."""
    f = lib().oracle_atan2f
    y, x = _c(y).ravel(), _c(x).ravel()
    return np.array([f(float(a), float(b)) for a, b in zip(y, x)], dtype=np.float32)


def tanf(x: np.ndarray) -> np.ndarray:
    """aaa_oracle.cpp oracle_tanf element-wise (the AAA bounds' tan)."""
    f = lib().oracle_tanf
    x = _c(x).ravel()
    return np.array([f(float(v)) for v in x], dtype=np.float32)


def cameras_prepare(views, Ks, width, height, with_centers):
    views, Ks = _c(views).reshape(-1, 16), _c(Ks).reshape(-1, 9)
    n = len(views)
    full = np.zeros((n, 16), np.float32)
    inverse = np.zeros((n, 16), np.float32)
    centers = np.zeros((n, 3), np.float32)
    errors = np.zeros(n, np.int32)
    lib().oracle_cameras_prepare(n, views, Ks, width, height, int(with_centers),
                                 _ptr(full), _ptr(inverse), _ptr(centers), errors)
    return full.reshape(n, 4, 4), inverse.reshape(n, 4, 4), centers, errors


def cameras_backward(Ks, grad_full, width, height, inverse, grad_centers):
    Ks = _c(Ks).reshape(-1, 9)
    n = len(Ks)
    gf = None if grad_full is None else _c(grad_full).reshape(n, 16)
    inv = None if inverse is None else _c(inverse).reshape(n, 16)
    gc = None if grad_centers is None else _c(grad_centers).reshape(n, 3)
    out = np.zeros((n, 16), np.float32)
    lib().oracle_cameras_backward(n, Ks, _ptr(gf), width, height, _ptr(inv), _ptr(gc), out)
    return out.reshape(n, 4, 4)


@dataclass
class Projected:
    centers: np.ndarray
    conics: np.ndarray
    radii: np.ndarray
    tiles: np.ndarray
    depths: np.ndarray


TILE_MODES = {"radius": 0, "snugbox": 1, "accutile": 2}


def project_forward(means, quats, scales, opacities, view, proj, K, width, height,
                    near=0.2, far=float("inf"), radius_clip=0.0, tile_mode="radius") -> Projected:
    n = len(means)
    out = Projected(np.zeros((n, 2), np.float32), np.zeros((n, 4), np.float32),
                    np.zeros(n, np.int32), np.zeros(n, np.int32), np.zeros(n, np.float32))
    lib().oracle_project_forward(
        n, _c(means), _c(quats), _c(scales), _c(opacities), _c(view).reshape(16),
        _c(proj).reshape(16), _c(K).reshape(9), width, height, near, far, radius_clip,
        out.centers, out.conics, out.radii, out.tiles, out.depths, TILE_MODES[tile_mode])
    return out


def sh_forward(coeffs, dirs, degree, radii=None):
    coeffs = _c(coeffs)
    n, K = coeffs.shape[0], coeffs.shape[1]
    colors = np.zeros((n, 3), np.float32)
    active = np.zeros((n, 3), np.uint8)
    r = None if radii is None else _c(radii, np.int32)
    lib().oracle_sh_forward(n, degree, K, coeffs, _c(dirs), _ptr(r), colors, _ptr(active))
    return colors, active


def sh_backward(coeffs, dirs, degree, radii, active, upstream, need_dirs=True):
    coeffs = _c(coeffs)
    n, K = coeffs.shape[0], coeffs.shape[1]
    gcoef = np.zeros_like(coeffs)
    gdir = np.zeros((n, 3), np.float32) if need_dirs else None
    r = None if radii is None else _c(radii, np.int32)
    lib().oracle_sh_backward(n, degree, K, coeffs, _c(dirs), _ptr(r), _c(active, np.uint8),
                             _c(upstream), gcoef, _ptr(gdir))
    return gcoef, gdir


def scan_counts(counts):
    counts = _c(counts, np.int32)
    offsets = np.zeros(len(counts), np.int32)
    m = lib().oracle_scan_counts(len(counts), counts, offsets)
    return offsets, int(m)


def bin_and_sort(centers, radii, depths, offsets, width, height, conics=None,
                 tile_mode="radius"):
    n = len(radii)
    m = int(offsets[-1]) if n else 0
    gx, gy = (width + 15) // 16, (height + 15) // 16
    keys = np.zeros(m, np.uint64)
    ids = np.zeros(m, np.int32)
    ranges = np.zeros((gx * gy, 2), np.int32)
    if tile_mode != "radius" and conics is None:
        raise ValueError("SnugBox/AccuTile require projected conics")
    conics_c = None if conics is None else _c(conics)  # alive across the call
    lib().oracle_bin_and_sort(n, _c(centers), _c(radii, np.int32), _c(depths),
                              _c(offsets, np.int32), width, height, keys, ids, ranges,
                              _ptr(conics_c), TILE_MODES[tile_mode])
    return keys, ids, ranges


def render_forward(width, height, ranges, ids, centers, conics, features, background):
    features = _c(features)
    c = features.shape[1]
    image = np.zeros((c, height, width), np.float32)
    final_t = np.zeros((height, width), np.float32)
    contrib = np.zeros((height, width), np.int32)
    lib().oracle_render_forward(width, height, c, _c(ranges, np.int32), _c(ids, np.int32),
                                _c(centers), _c(conics), features, _c(background), image,
                                final_t, contrib)
    return image, final_t, contrib


def render_backward(width, height, ranges, ids, centers, conics, features, background,
                    final_t, contributors, upstream, absgrad=False, constant_tail=0):
    """upstream: planar (C,H,W).  Returns float64 accumulators."""
    features = _c(features)
    n, c = features.shape
    gc = np.zeros((n, 2), np.float64)
    gq = np.zeros((n, 4), np.float64)
    gf = np.zeros((n, c), np.float64)
    ga = np.zeros((n, 2), np.float64) if absgrad else None
    lib().oracle_render_backward(width, height, c, constant_tail, _c(ranges, np.int32),
                                 _c(ids, np.int32), _c(centers), _c(conics), features,
                                 _c(background), _c(final_t), _c(contributors, np.int32),
                                 _c(upstream), gc, gq, gf, _ptr(ga))
    return gc, gq, gf, ga


def project_backward(means, quats, scales, opacities, view, proj, K, width, height, radii,
                     seed_centers, seed_conics):
    n = len(means)
    gm = np.zeros((n, 3), np.float32)
    gq = np.zeros((n, 4), np.float32)
    gs = np.zeros((n, 3), np.float32)
    go = np.zeros(n, np.float32)
    gv = np.zeros(16, np.float64)
    gp = np.zeros(16, np.float64)
    lib().oracle_project_backward(
        n, _c(means), _c(quats), _c(scales), _c(opacities), _c(view).reshape(16),
        _c(proj).reshape(16), _c(K).reshape(9), width, height, _c(radii, np.int32),
        _c(seed_centers), _c(seed_conics), gm, gq, gs, go, _ptr(gv), _ptr(gp))
    return gm, gq, gs, go, gv.reshape(4, 4), gp.reshape(4, 4)


# --------------------------------------------------------------------------
# One gs3d view end to end: gs3d/api.py:47-265 + gs3d/autograd.py:19-171 for a
# single camera, composed from the stage functions above.


@dataclass
class ViewResult:
    image: np.ndarray          # (C', H, W) planar, C' = channels + extras + 1
    final_t: np.ndarray
    contributors: np.ndarray
    proj: Projected
    keys: np.ndarray
    ids: np.ndarray
    ranges: np.ndarray
    features: np.ndarray       # (N, C') blended attributes
    colors_active: np.ndarray | None
    full: np.ndarray
    inverse: np.ndarray
    campos: np.ndarray | None


def gs3d_view_forward(means, quats_n, scales, opacities, viewmat, K, width, height, *,
                      sh_coeffs=None, sh_degree=None, features=None, extras=None,
                      background=None, near=0.2, far=float("inf"), radius_clip=0.0,
                      tile_mode="radius"):
    """quats_n must already be normalised (the reference normalises with Torch)."""
    with_centers = sh_coeffs is not None and sh_degree > 0
    full, inverse, campos, errors = cameras_prepare(viewmat[None], K[None], width, height,
                                                    with_centers)
    if errors[0]:
        raise ValueError(f"camera error code {errors[0]}")
    p = project_forward(means, quats_n, scales, opacities, viewmat, full[0], K, width,
                        height, near, far, radius_clip, tile_mode=tile_mode)
    active = None
    if sh_coeffs is not None:
        dirs = (np.asarray(means, np.float32) - campos[0][None]) if with_centers else np.asarray(means, np.float32)
        colors, active = sh_forward(sh_coeffs, dirs, sh_degree, p.radii)
    else:
        colors = np.asarray(features, np.float32)
    cols = [colors]
    if extras is not None:
        cols.append(np.asarray(extras, np.float32))
    cols.append(np.ones((len(means), 1), np.float32))
    attrs = np.ascontiguousarray(np.concatenate(cols, axis=1), dtype=np.float32)
    bg = np.zeros(attrs.shape[1], np.float32)
    if background is not None:
        bg[: colors.shape[1]] = background
    offsets, m = scan_counts(p.tiles)
    keys, ids, ranges = bin_and_sort(p.centers, p.radii, p.depths, offsets, width, height,
                                     conics=p.conics, tile_mode=tile_mode)
    image, final_t, contrib = render_forward(width, height, ranges, ids, p.centers, p.conics,
                                             attrs, bg)
    return ViewResult(image, final_t, contrib, p, keys, ids, ranges, attrs, active, full[0],
                      inverse[0], None if not with_centers else campos[0]), bg


@dataclass
class ViewGrads:
    means: np.ndarray
    quats_n: np.ndarray        # w.r.t. the normalised quaternions
    scales: np.ndarray
    opacities: np.ndarray
    sh: np.ndarray | None
    colors: np.ndarray | None  # features path
    extras: np.ndarray | None
    viewmat: np.ndarray
    means2d: np.ndarray
    absgrad: np.ndarray


def gs3d_view_backward(r: ViewResult, bg, means, quats_n, scales, opacities, viewmat, K, width,
                       height, upstream_hwc, *, sh_coeffs=None, sh_degree=None, n_colors=3,
                       n_extras=0):
    """Reverse of gs3d_view_forward: gs3d/autograd.py:91-171 + SH + camera VJPs."""
    up = np.ascontiguousarray(np.moveaxis(np.asarray(upstream_hwc, np.float32), -1, 0))
    gc, gq, gf, ga = render_backward(width, height, r.ranges, r.ids, r.proj.centers,
                                     r.proj.conics, r.features, bg, r.final_t, r.contributors,
                                     up, absgrad=True, constant_tail=1)
    gm, gqn, gs, go, gview, gproj = project_backward(
        means, quats_n, scales, opacities, viewmat, r.full, K, width, height, r.proj.radii,
        gc.astype(np.float32), gq.astype(np.float32))
    gm = gm.astype(np.float64)
    gcolor = gf[:, :n_colors]
    gsh = None
    gcampos = None
    if sh_coeffs is not None:
        with_centers = sh_degree > 0
        dirs = (np.asarray(means, np.float32) - r.campos[None]) if with_centers else np.asarray(means, np.float32)
        gsh, gdir = sh_backward(sh_coeffs, dirs, sh_degree, r.proj.radii, r.colors_active,
                                gcolor.astype(np.float32), need_dirs=with_centers)
        if with_centers:
            gm = gm + gdir
            gcampos = -gdir.astype(np.float64).sum(0)
    gv_cam = cameras_backward(K[None], gproj[None].astype(np.float32), width, height,
                              r.inverse[None] if gcampos is not None else None,
                              None if gcampos is None else gcampos[None].astype(np.float32))[0]
    return ViewGrads(gm, gqn, gs, go, gsh, None if sh_coeffs is not None else gcolor,
                     gf[:, n_colors:n_colors + n_extras] if n_extras else None,
                     gview + gv_cam.astype(np.float64), gc, ga)


# ---- RaDe-GS ---------------------------------------------------------------

def rade_project(means, quats, scales, opacities, view, proj, K, width, height, *,
                 near=0.2, far=float("inf"), radius_clip=0.0, kernel_size=0.0):
    """rade/projection.py:194-260: centers, conics, radii, tiles, depths,
    planes, normals (culled rows zero)."""
    means = _c(means).reshape(-1, 3)
    n = len(means)
    out = dict(centers=np.zeros((n, 2), np.float32), conics=np.zeros((n, 4), np.float32),
               radii=np.zeros(n, np.int32), tiles=np.zeros(n, np.int32),
               depths=np.zeros(n, np.float32), planes=np.zeros((n, 3), np.float32),
               normals=np.zeros((n, 3), np.float32))
    lib().oracle_rade_project(
        n, means, _c(quats), _c(scales), _c(opacities), _c(view), _c(proj), _c(K), width, height,
        near, far, radius_clip, kernel_size, out["centers"], out["conics"], out["radii"],
        out["tiles"], out["depths"], out["planes"], out["normals"])
    return out


def rade_render(width, height, ranges, ids, centers, conics, features, background, planes,
                normals, K):
    """rade/render.py:106-227: image (C+6,H,W), auxiliary (2,H,W), contributors (2,H,W)."""
    features = _c(features)
    C = features.shape[1]
    image = np.zeros((C + 6, height, width), np.float32)
    aux = np.zeros((2, height, width), np.float32)
    contrib = np.zeros((2, height, width), np.int32)
    lib().oracle_rade_render(width, height, C, _c(ranges, np.int32), _c(ids, np.int32),
                             _c(centers), _c(conics), features, _c(background), _c(planes),
                             _c(normals), _c(K), image, aux, contrib)
    return image, aux, contrib


def rade_render_backward(width, height, ranges, ids, centers, conics, features, background,
                         planes, normals, K, image, aux, contrib, up_features=None,
                         up_alpha=None, up_depth=None, up_median=None, up_normals=None,
                         absgrad=True):
    """rade/render.py:336-545; upstream images channel-last (H,W,k) or None.
    Returns float64 grads of centers, conics, features, |centers|, planes, normals."""
    features = _c(features)
    n, C = features.shape
    g = dict(centers=np.zeros((n, 2)), conics=np.zeros((n, 4)), features=np.zeros((n, C)),
             abs=np.zeros((n, 2)) if absgrad else None, planes=np.zeros((n, 3)),
             normals=np.zeros((n, 3)))
    ups = [None if u is None else _c(u) for u in (up_features, up_alpha, up_depth, up_median,
                                                   up_normals)]
    lib().oracle_rade_render_backward(
        width, height, C, _c(ranges, np.int32), _c(ids, np.int32), _c(centers), _c(conics),
        features, _c(background), _c(planes), _c(normals), _c(K), _c(image), _c(aux),
        _c(contrib, np.int32), *[_ptr(u) for u in ups], g["centers"], g["conics"],
        g["features"], _ptr(g["abs"]), g["planes"], g["normals"])
    return g


AAA_FLAGS = ("ewa", "new_aabb", "near_clipping", "tile_culling", "complete", "cooperative")


def aaa_preprocess(means, quats, scales, opacities, view, proj, campos, width, height,
                   tanfov, principal, *, sh=None, sh_degree=0, filters=None, sort_order=3,
                   modifier=1.0, flags=None):
    """aaa/preprocess3d.py:17-245 for one view (aaa_oracle.cpp).

    view / proj are the reference's transposed 4x4 camera arrays
    (aaa/cameras.py:77-121); flags maps AAA_FLAGS to bools (default: the
    load-balanced path of aaa/config.py:41-54).  Returns the geometry rows,
    radii / tiles / valid, the colours when sh is given, and the sorted
    indices of the Gaussians queued for the collective cull."""
    flags = dict(dict(ewa=True, new_aabb=True, near_clipping=False, tile_culling=True,
                      complete=False, cooperative=True), **(flags or {}))
    n = len(means)
    use_sh = sh is not None
    sh_c = _c(sh) if use_sh else None
    K = sh_c.shape[1] if use_sh else 0
    filt = _c(filters) if filters is not None else None
    out = dict(centers=np.zeros((n, 2), np.float32), rects=np.zeros((n, 2), np.float32),
               depths=np.zeros(n, np.float32), transforms=np.zeros((n, 4, 4), np.float32),
               opacity=np.zeros(n, np.float32), radii=np.zeros(n, np.int32),
               tiles=np.zeros(n, np.int32), valid=np.zeros(n, np.uint8))
    rgb = np.zeros((n, 3), np.float32) if use_sh else None
    clamped = np.zeros((n, 3), np.uint8) if use_sh else None
    queued = np.full(max(n, 1), -1, np.int32)
    size = np.zeros(1, np.int32)
    lib().oracle_aaa_preprocess(
        n, _c(means), _c(scales), _c(quats), _c(opacities), _ptr(sh_c), K, int(use_sh),
        int(sh_degree), int(sort_order), _ptr(filt), _c(campos), _c(view), _c(proj),
        int(width), int(height), float(tanfov[0]), float(tanfov[1]), float(principal[0]),
        float(principal[1]), float(modifier), *[int(bool(flags[k])) for k in AAA_FLAGS],
        out["centers"], out["rects"], out["depths"], out["transforms"], out["opacity"],
        out["radii"], out["tiles"], _ptr(rgb), out["valid"], _ptr(clamped), queued, size)
    out["valid"] = out["valid"].astype(bool)
    if use_sh:
        out["rgb"], out["clamped"] = rgb, clamped.astype(bool)
    out["queued"] = np.sort(queued[:size[0]])
    return out


def aaa_cull_remainder(pre: dict, width: int, height: int) -> dict:
    """aaa/cooperative_culling.py:152-192 on aaa_preprocess's output: the
    final radii / tiles / valid of the load-balanced path (new arrays)."""
    radii, tiles = pre["radii"].copy(), pre["tiles"].copy()
    valid = pre["valid"].astype(np.uint8)
    q = _c(pre["queued"], np.int32)
    lib().oracle_aaa_cull_remainder(
        q, len(q), _c(pre["centers"]), _c(pre["rects"]), _c(pre["transforms"]),
        _c(pre["opacity"]), int(width), int(height), radii, tiles, valid)
    return dict(radii=radii, tiles=tiles, valid=valid.astype(bool))


def aaa_duplicate(pre: dict, radii, tiles, width: int, height: int, offsets=None):
    """aaa/binning_native.py:7-135 (aaa_oracle.cpp): keys and Gaussian ids of
    every visible Gaussian's tiles.  offsets defaults to the inclusive scan of
    the visible Gaussians' tile counts; returns (offsets, keys, values)."""
    radii = _c(radii, np.int32)
    if offsets is None:
        offsets = np.cumsum(np.where(radii > 0, tiles, 0)).astype(np.int32)
    offsets = _c(offsets, np.int32)
    total = int(offsets[-1]) if len(offsets) else 0
    keys = np.zeros(total, np.uint64)
    values = np.full(total, -7, np.int32)
    lib().oracle_aaa_duplicate(
        len(radii), _c(pre["centers"]), _c(pre["rects"]), radii, _c(pre["transforms"]),
        _c(pre["opacity"]), offsets, int(width), int(height), keys, values, total)
    return offsets, keys, values


def aaa_preprocess_backward(means, quats, scales, opacities, radii, view, proj, campos, width,
                            height, focal_x, up_transforms, up_opacity, *, ewa=True):
    """aaa/backward_preprocess.py:130-268 (aaa_oracle.cpp): the gradients of
    the opacities, means, scales and quaternions from the gradients of the
    Gaussian-to-screen transforms and effective opacities."""
    n = len(means)
    out = dict(opacity=np.zeros(n, np.float32), means=np.zeros((n, 3), np.float32),
               scales=np.zeros((n, 3), np.float32), quats=np.zeros((n, 4), np.float32))
    lib().oracle_aaa_preprocess_backward(
        n, _c(means), _c(scales), _c(quats), _c(opacities), _c(radii, np.int32), _c(view),
        _c(proj), _c(campos), int(width), int(height), float(focal_x), int(bool(ewa)),
        _c(up_transforms), _c(up_opacity), out["opacity"], out["means"], out["scales"],
        out["quats"])
    return out


def aaa_camera_backward(means, quats, scales, radii, effective_opacity, view, proj, campos,
                        width, height, focal, up_transforms, up_opacity, up_colors, *,
                        filters=None, sh=None, sh_degree=0, clamped=None, ewa=True,
                        modifier=1.0):
    """aaa/backward_camera.py:61-224 (aaa_oracle.cpp): per-Gaussian (n, 23)
    camera-gradient rows (the reference sums them over Gaussians)."""
    n = len(means)
    rows = np.zeros((n, 23), np.float32)
    sh_c = _c(sh) if sh is not None else None
    cl = _c(clamped, np.uint8) if sh is not None else None
    filt = _c(filters) if filters is not None else None
    lib().oracle_aaa_camera_backward(
        n, _c(means), _c(scales), _c(quats), _ptr(filt), _c(radii, np.int32),
        _c(effective_opacity), _c(view), _c(proj), _c(campos), int(width), int(height),
        float(focal), float(modifier), int(bool(ewa)), _c(up_transforms), _c(up_opacity),
        _ptr(sh_c), sh_c.shape[1] if sh_c is not None else 0, int(sh_degree), _ptr(cl),
        _c(up_colors), rows)
    return rows


def aaa_sort(keys, values, tiles_total):
    """primitives/tiling.py:67-100 on AAA keys: a stable sort of the pairs on
    key bits [0, 32 + bit_length(T)) (Warp's radix_sort_pairs end_bit; the
    padding tile 0xffffffff then sorts after every real tile), and the tile
    ranges of identify_ranges (:39-54), which skips the padding tile."""
    keys = np.asarray(keys, np.uint64)
    end_bit = 32 + int(tiles_total).bit_length()
    masked = keys & np.uint64((1 << end_bit) - 1)
    order = np.argsort(masked, kind="stable")
    skeys, svals = keys[order], np.asarray(values, np.int32)[order]
    ranges = np.zeros((tiles_total, 2), np.int32)
    tile = (skeys >> np.uint64(32)).astype(np.int64)
    real = tile != 0xFFFFFFFF
    if real.any():
        idx = np.nonzero(real)[0]
        t = tile[idx]
        starts = np.r_[True, t[1:] != t[:-1]]
        ends = np.r_[t[1:] != t[:-1], True]
        ranges[t[starts], 0] = idx[starts]
        ranges[t[ends], 1] = idx[ends] + 1
    return skeys, svals, ranges


def aaa_render(width, height, ranges, points, transforms, opacity, colors, bg, cull=True,
               stat_maps=None, stat_kinds=()):
    """aaa/render_hierarchical_warp.py:599-691 (aaa_render_oracle.cpp): the
    HIER 64/8/4 blend.  Returns image (C, H, W), final_t (H, W) and the
    evaluated-sample counts (H, W); with stat_maps ((R, H, W), kinds 0 =
    masked count, 1 = weighted sum) also the statistics: counts (Rc, n)
    int32 and float64 sums (Rs, n) (statistics.py:47-73)."""
    colors = _c(colors)
    n, C = colors.shape
    image = np.zeros((C, height, width), np.float32)
    final_t = np.zeros((height, width), np.float32)
    contrib = np.zeros((height, width), np.int32)
    kinds = tuple(stat_kinds)
    maps = (np.zeros((1, 1), np.float32) if stat_maps is None
            else _c(np.asarray(stat_maps, np.float32).reshape(len(kinds), -1)))
    counts = np.zeros((max(1, kinds.count(0)), n), np.int32)
    sums = np.zeros((max(1, kinds.count(1)), n), np.float64)
    mask = sum(1 << r for r, k in enumerate(kinds) if k == 1)
    assert lib().oracle_aaa_render(
        int(width), int(height), C, _c(ranges, np.int32), _c(points, np.int32),
        _c(transforms), _c(opacity), colors, _c(bg), int(bool(cull)), image, final_t,
        contrib, n, len(kinds) if stat_maps is not None else 0, mask, maps, counts, sums) == 0
    if stat_maps is None:
        return image, final_t, contrib
    return image, final_t, contrib, counts[: kinds.count(0)], sums[: kinds.count(1)]


def aaa_render_backward(width, height, ranges, points, transforms, opacity, colors, bg, image,
                        final_t, pixel_grad, cull=True, screen=False, absgrad=False):
    """aaa/backward_render.py:75-248 (aaa_render_oracle.cpp): float64 sums of
    the replay's gradients -- transforms (n, 16) in the reference's transposed
    layout, opacity (n), colours (n, C), and the optional screen-translation
    statistics (n, 2) and their absolute sums (n, 2)."""
    colors = _c(colors)
    n, C = colors.shape
    out = dict(transforms=np.zeros((n, 16)), opacity=np.zeros(n), colors=np.zeros((n, C)))
    scr = np.zeros((n, 2)) if screen else None
    sabs = np.zeros((n, 2)) if screen and absgrad else None
    assert lib().oracle_aaa_render_backward(
        int(width), int(height), C, _c(ranges, np.int32), _c(points, np.int32),
        _c(transforms), _c(opacity), colors, _c(bg), int(bool(cull)), _c(image), _c(final_t),
        _c(pixel_grad), out["transforms"], out["opacity"], out["colors"], _ptr(scr),
        _ptr(sabs)) == 0
    if screen:
        out["screen"] = scr
    if absgrad:
        out["screen_abs"] = sabs
    return out
