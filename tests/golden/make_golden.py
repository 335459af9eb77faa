"""Generate golden vectors from dsl_splat's own gs3d kernels (test infrastructure).

Runs where a dsl_splat checkout is available (its root as argv[1] or in the
DSL_SPLAT_REFERENCE environment variable); the committed .npz files are what the tests
read, so nothing at test time needs the reference.  warp-lang is absent, so
the reference modules are imported with warp_shim registered as `warp` (see
that module for exactly what is emulated and the one substitution, exp).

Kernels executed (reference file:line):
  splatting/camera_kernels.py:11-66   prepare_kernel
  splatting/camera_kernels.py:69-106  backward_kernel
  gs3d/projection.py:89-164           project (tile_mode "radius")
  primitives/sh.py:44-79, 82-138      SH forward / backward kernels
  splatting/metadata.py:12-31         _prepare
  splatting/binning.py:16-37        duplicate
  primitives/tiling.py:39-54          identify_ranges
  gs3d/render.py:36-208               render (forward blend, 256-thread blocks)
  gs3d/render.py:211-356              backward (reverse blend, 256-thread blocks)
Warp library calls restated: array_scan (inclusive cumsum) and
radix_sort_pairs (a stable sort of the 64-bit keys).

Also: gs3d/render.py:36-208 with statistics.py:47-73's observer and eight
channels (wide_*.npz); and the RaDe-GS path (rade_*.npz):
  rade/projection.py:194-260          project (ray planes, normals, radial depth,
                                      kernel_size dilation)
  splatting/binning.py:16-37        duplicate with the radial depths
  rade/render.py:99-322               render (colour, depth, median, normals)
  rade/render.py:325-547              backward (warp-reduced atomics)

And the AAA-Gaussians preprocessing (aaa_*.npz), cameras lowered by
aaa/cameras.py:77-121 (prepare_cameras) and Gaussians run through
  aaa/preprocess3d.py:17-245          preprocess_3d (adaptive 3D filter,
                                      perspective-correct bounds, tile culling,
                                      long-rectangle queue)
  aaa/cooperative_culling.py:152-192  cull_remainder_3d (the queued rectangles'
                                      tiles past the first 32, 32-lane tile_sum;
                                      final_* keys of the load-balanced cases)
  aaa/binning_native.py:7-135         duplicate_aaa_default (the warp-cooperative
                                      key emission, its snippet compiled with the
                                      shim's 32-thread warp lanes; dup_* keys of
                                      aaa_coop)
  aaa/backward_preprocess.py:130-268  preprocess_adjoint (seeded N(0,1) transform
                                      and opacity upstreams; adj_* keys)
  aaa/backward_camera.py:61-224       camera_adjoint (the same upstreams and a
                                      seeded colour gradient; cam_* keys, the
                                      per-Gaussian 23-float rows)
with aaa/native_geometry.py's snippets (frustum depth, axis bounds, screen
bounds) compiled by g++ against the host libm (atan2f, tanf, fmodf).

Usage: python tests/golden/make_golden.py [/path/to/reference]
       [--tile-modes-only | --wide-only | --rade-only | --aaa-only]
"""

from __future__ import annotations

import ctypes
import importlib
import os
import sys
import time
import types

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, ROOT)

import warp_shim as ws  # noqa: E402


def load_reference(ref_root: str):
    sys.modules["warp"] = ws.make_module()
    pkg_root = os.path.join(ref_root, "dsl_splat")
    # Stub the packages so their __init__ files (which import the AAA stack)
    # are not executed; submodules load from the checkout.
    for pkg in ("dsl_splat", "dsl_splat.gs3d", "dsl_splat.splatting", "dsl_splat.primitives",
                "dsl_splat.runtime", "dsl_splat.rade", "dsl_splat.aaa"):
        mod = types.ModuleType(pkg)
        parts = pkg.split(".")[1:]
        mod.__path__ = [os.path.join(pkg_root, *parts)]
        sys.modules[pkg] = mod
    from oracle import oracle as O
    ws.set_exp(lambda x: np.float32(O.lib().oracle_expf(float(x))))
    ws.set_log(lambda x: np.float32(O.lib().oracle_logf(float(x))))
    names = {
        "cam": "dsl_splat.splatting.camera_kernels",
        "proj": "dsl_splat.gs3d.projection",
        "sh": "dsl_splat.primitives.sh",
        "meta": "dsl_splat.splatting.metadata",
        "bin": "dsl_splat.splatting.binning",
        "tiling": "dsl_splat.primitives.tiling",
        "render": "dsl_splat.gs3d.render",
        "rade_proj": "dsl_splat.rade.projection",
        "rade_render": "dsl_splat.rade.render",
    }
    return {k: importlib.import_module(v) for k, v in names.items()}


def A(data, dtype=None):
    return ws.Array(data, dtype)


def golden_case(ref, name, scene: dict, seed: int):
    W, H = scene["width"], scene["height"]
    gx, gy = (W + 15) // 16, (H + 15) // 16
    T = gx * gy
    deg = scene["sh_degree"]
    means = scene["means"].astype(np.float32)
    n = len(means)
    quats_raw = scene["quats"].astype(np.float32)
    quats = F.normalize(torch.from_numpy(quats_raw), dim=-1).numpy()  # inputs.py:252
    scales = scene["scales"].astype(np.float32)
    opac = scene["opacities"].astype(np.float32)
    sh = scene["sh"].astype(np.float32)
    view = scene["viewmat"].astype(np.float32)
    K = scene["K"].astype(np.float32)
    wp = sys.modules["warp"]
    out: dict = dict(width=W, height=H, sh_degree=deg, means=means, quats=quats, scales=scales,
                     opacities=opac, sh=sh, viewmat=view, K=K)
    t0 = time.time()

    # camera_kernels.py:11-66 (with centres: SH degree > 0 needs them)
    full = np.zeros((1, 4, 4), np.float32)
    inverse = np.zeros((1, 4, 4), np.float32)
    centers_cam = np.zeros((1, 3), np.float32)
    errors = np.zeros(1, np.int32)
    ws.launch(ref["cam"].prepare_kernel, 1,
              [A(view[None].copy()), A(K[None].copy()), W, H, 1, A(full), A(inverse),
               A(centers_cam), A(errors)])
    assert errors[0] == 0
    out.update(full=full[0], inverse=inverse[0], campos=centers_cam[0])

    # gs3d/projection.py:89-164
    centers = np.zeros((n, 2), np.float32)
    conics = np.zeros((n, 4), np.float32)
    radii = np.zeros(n, np.int32)
    tiles = np.zeros(n, np.int32)
    depths = np.zeros(n, np.float32)
    ws.launch(ref["proj"].project, n,
              [A(means, wp.vec3), A(quats, wp.vec4), A(scales, wp.vec3), A(opac), A(view.copy()),
               A(full[0].copy()), A(K.copy()), W, H, np.float32(0.2), np.float32(np.inf),
               np.float32(0.0), A(centers, wp.vec2), A(conics, wp.vec4), A(radii), A(tiles),
               A(depths)])
    out.update(centers=centers, conics=conics, radii=radii, tiles=tiles, depths=depths)

    # primitives/sh.py:44-79 masked forward with saved clamp mask; directions
    # are the Torch difference means - camera centre (gs3d/api.py:158-168)
    dirs = (torch.from_numpy(means) - torch.from_numpy(centers_cam[0])).numpy()
    colors = np.zeros((n, 3), np.float32)
    active = np.zeros((n, 3), np.bool_)
    ws.launch(ref["sh"].forward_kernel(deg, True, True), n,
              [A(sh), A(dirs), A(radii), A(colors, wp.vec3), A(active)])
    out.update(dirs=dirs, colors=colors, active=active)

    # splatting/metadata.py:12-31
    m2d = np.zeros((n, 2), np.float32)
    mop = np.zeros(n, np.float32)
    mcon = np.zeros((n, 3), np.float32)
    ws.launch(ref["meta"]._prepare, n, [A(radii), A(centers, wp.vec2), A(conics, wp.vec4),
                                         A(m2d, wp.vec2), A(mop), A(mcon, wp.vec3)])
    out.update(meta_means2d=m2d, meta_opacities=mop, meta_conics=mcon)

    # primitives/tiling.py:57-64 (Warp array_scan, inclusive) and
    # splatting/binning.py:16-37 duplicate
    offsets = np.cumsum(tiles, dtype=np.int64).astype(np.int32)
    m = int(offsets[-1]) if n else 0
    keys = np.zeros(2 * m, np.uint64)
    ids = np.zeros(2 * m, np.int32)
    ws.launch(ref["bin"].duplicate, n, [A(centers, wp.vec2), A(radii), A(depths), A(offsets),
                                         gx, gy, A(keys), A(ids)])
    # primitives/tiling.py:80-86 (Warp radix_sort_pairs: a stable LSD sort)
    order = np.argsort(keys[:m], kind="stable")
    keys_sorted = keys[:m][order]
    ids_sorted = ids[:m][order]
    ranges = np.zeros((T, 2), np.int32)
    ws.launch(ref["tiling"].identify_ranges, m, [A(keys_sorted), A(ranges)])
    out.update(offsets=offsets, keys=keys_sorted, ids=ids_sorted, ranges=ranges)

    # gs3d/autograd.py:42-46: features = cat(colours, ones); black background
    feats = np.concatenate([colors, np.ones((n, 1), np.float32)], axis=1)
    C = feats.shape[1]
    bg = np.zeros(C, np.float32)
    Feature = wp.types.vector(C, np.float32)
    image = np.zeros(C * H * W, np.float32)
    final_t = np.zeros(H * W, np.float32)
    contrib = np.zeros(H * W, np.int32)
    ws.launch(ref["render"]._make_forward(C, ()), 256 * T,
              [W, H, A(ranges), A(ids_sorted), A(centers, wp.vec2), A(conics, wp.vec4),
               A(feats, Feature), A(bg), A(image), A(final_t), A(contrib)], block=256)
    out.update(features=feats, background=bg, image=image.reshape(C, H, W),
               final_t=final_t.reshape(H, W), contributors=contrib.reshape(H, W))

    # gs3d/render.py:211-356 backward, absgrad, constant alpha tail
    rng = np.random.default_rng(seed)
    upstream = rng.standard_normal((C, H, W)).astype(np.float32)
    g_centers = np.zeros((n, 2), np.float32)
    g_conics = np.zeros((n, 4), np.float32)
    g_feats = np.zeros((n, C), np.float32)
    g_abs = np.zeros((n, 2), np.float32)
    ws.launch(ref["render"]._make_backward(C, True, 1), 256 * T,
              [W, H, A(ranges), A(ids_sorted), A(centers, wp.vec2), A(conics, wp.vec4),
               A(feats, Feature), A(bg), A(final_t), A(contrib), A(upstream.ravel().copy()),
               A(g_centers), A(g_conics), A(g_feats), A(g_abs)], block=256)
    out.update(upstream=upstream, grad_centers=g_centers, grad_conics=g_conics,
               grad_features=g_feats, grad_abs=g_abs)

    # primitives/sh.py:82-138 backward with the blended colour gradient
    g_sh = np.zeros_like(sh)
    g_dirs = np.zeros((n, 3), np.float32)
    up_colors = g_feats[:, :3].copy()
    ws.launch(ref["sh"].backward_kernel(deg, True, True, deg > 0), n,
              [A(sh), A(dirs), A(radii), A(active), A(up_colors), A(g_sh), A(g_dirs, wp.vec3)])
    out.update(sh_upstream=up_colors, grad_sh=g_sh, grad_dirs=g_dirs)

    # splatting/camera_kernels.py:69-106 pose VJP through full and the centre
    gfull = rng.standard_normal((1, 4, 4)).astype(np.float32)
    gcam = rng.standard_normal((1, 3)).astype(np.float32)
    gviews = np.zeros((1, 4, 4), np.float32)
    ws.launch(ref["cam"].backward_kernel, 1,
              [A(K[None].copy()), A(gfull), W, H, A(inverse), A(gcam), 1, 1, A(gviews)])
    out.update(cam_grad_full=gfull[0], cam_grad_centers=gcam[0], cam_grad_views=gviews[0])
    print(f"{name}: n={n} visible={int((radii > 0).sum())} pairs={m} tiles={T} "
          f"in {time.time() - t0:.1f}s", flush=True)
    return out


def wide_case(ref, name, scene: dict, seed: int) -> dict:
    """Eight blended channels (3 SH colours, 4 extras, the constant one) over
    a random background, with one masked-count and one weighted-sum
    statistics request, through the reference's own render kernels
    (gs3d/render.py:36-208 with statistics.py:47-73's observer, and
    gs3d/render.py:211-356), on the projection and bins of `scene`."""
    base = golden_case(ref, name, scene, seed)
    W, H = base["width"], base["height"]
    T = ((W + 15) // 16) * ((H + 15) // 16)
    n = len(base["means"])
    wp = sys.modules["warp"]
    rng = np.random.default_rng(seed + 1000)
    extras = rng.standard_normal((n, 4)).astype(np.float32)
    feats = np.concatenate([base["colors"], extras, np.ones((n, 1), np.float32)], axis=1)
    C = feats.shape[1]
    bg = rng.uniform(0.0, 1.0, C).astype(np.float32)
    Feature = wp.types.vector(C, np.float32)
    mask = np.zeros((H, W), np.float32)
    mask[: H // 2] = 1.0
    weights = rng.uniform(0.0, 1.0, (H, W)).astype(np.float32)
    pixel_values = np.stack([mask.ravel(), weights.ravel()])  # request 0 count, 1 sum
    counts = np.zeros((1, n), np.int32)
    sums = np.zeros((1, n), np.float32)
    image = np.zeros(C * H * W, np.float32)
    final_t = np.zeros(H * W, np.float32)
    contrib = np.zeros(H * W, np.int32)
    ws.launch(ref["render"]._make_forward(C, (0, 1)), 256 * T,
              [W, H, A(base["ranges"]), A(base["ids"]), A(base["centers"], wp.vec2),
               A(base["conics"], wp.vec4), A(feats, Feature), A(bg), A(image), A(final_t),
               A(contrib), A(pixel_values), A(counts), A(sums)], block=256)
    upstream = rng.standard_normal((C, H, W)).astype(np.float32)
    g_centers = np.zeros((n, 2), np.float32)
    g_conics = np.zeros((n, 4), np.float32)
    g_feats = np.zeros((n, C), np.float32)
    g_abs = np.zeros((n, 2), np.float32)
    ws.launch(ref["render"]._make_backward(C, True, 1), 256 * T,
              [W, H, A(base["ranges"]), A(base["ids"]), A(base["centers"], wp.vec2),
               A(base["conics"], wp.vec4), A(feats, Feature), A(bg), A(final_t), A(contrib),
               A(upstream.ravel().copy()), A(g_centers), A(g_conics), A(g_feats), A(g_abs)],
              block=256)
    keep = {k: base[k] for k in ("width", "height", "centers", "conics", "radii", "ranges",
                                 "ids")}
    keep.update(features=feats, background=bg, mask=mask, weights=weights,
                image=image.reshape(C, H, W), final_t=final_t.reshape(H, W),
                contributors=contrib.reshape(H, W), stat_counts=counts[0], stat_sums=sums[0],
                upstream=upstream, grad_centers=g_centers, grad_conics=g_conics,
                grad_features=g_feats, grad_abs=g_abs)
    print(f"{name} (8 channels, statistics): pairs={len(base['ids'])}", flush=True)
    return keep


def rade_case(ref, name, scene: dict, seed: int, kernel_size: float, extra: int) -> dict:
    """RaDe-GS projection, radial-depth binning, render and render backward
    through the reference's own kernels, with SH colours (primitives/sh.py
    forward, as rade/api.py:153-165 calls it) plus `extra` N(0,1) channels
    and a random background over them."""
    W, H = scene["width"], scene["height"]
    gx, gy = (W + 15) // 16, (H + 15) // 16
    T = gx * gy
    deg = scene["sh_degree"]
    means = scene["means"].astype(np.float32)
    n = len(means)
    quats = F.normalize(torch.from_numpy(scene["quats"].astype(np.float32)), dim=-1).numpy()
    scales = scene["scales"].astype(np.float32)
    opac = scene["opacities"].astype(np.float32)
    sh = scene["sh"].astype(np.float32)
    view = scene["viewmat"].astype(np.float32)
    K = scene["K"].astype(np.float32)
    wp = sys.modules["warp"]
    t0 = time.time()
    full = np.zeros((1, 4, 4), np.float32)
    inverse = np.zeros((1, 4, 4), np.float32)
    campos = np.zeros((1, 3), np.float32)
    errors = np.zeros(1, np.int32)
    ws.launch(ref["cam"].prepare_kernel, 1,
              [A(view[None].copy()), A(K[None].copy()), W, H, 1, A(full), A(inverse),
               A(campos), A(errors)])
    assert errors[0] == 0
    ks = np.float32(kernel_size)
    out: dict = dict(width=W, height=H, sh_degree=deg, means=means, quats=quats,
                     scales=scales, opacities=opac, sh=sh, viewmat=view, K=K, full=full[0],
                     campos=campos[0], kernel_size=ks)

    # rade/projection.py:194-260
    centers = np.zeros((n, 2), np.float32)
    conics = np.zeros((n, 4), np.float32)
    radii = np.zeros(n, np.int32)
    tiles = np.zeros(n, np.int32)
    depths = np.zeros(n, np.float32)
    planes = np.zeros((n, 3), np.float32)
    normals = np.zeros((n, 3), np.float32)
    ws.launch(ref["rade_proj"].project, n,
              [A(means, wp.vec3), A(quats, wp.vec4), A(scales, wp.vec3), A(opac),
               A(view.copy()), A(full[0].copy()), A(K.copy()), W, H, np.float32(0.2),
               np.float32(np.inf), np.float32(0.0), ks, A(centers, wp.vec2),
               A(conics, wp.vec4), A(radii), A(tiles), A(depths), A(planes, wp.vec3),
               A(normals, wp.vec3)])
    out.update(centers=centers, conics=conics, radii=radii, tiles=tiles, depths=depths,
               planes=planes, normals=normals)

    # colours: primitives/sh.py:44-79 with directions means - camera centre
    dirs = (torch.from_numpy(means) - torch.from_numpy(campos[0])).numpy()
    colors = np.zeros((n, 3), np.float32)
    active = np.zeros((n, 3), np.bool_)
    ws.launch(ref["sh"].forward_kernel(deg, True, True), n,
              [A(sh), A(dirs), A(radii), A(colors, wp.vec3), A(active)])
    rng = np.random.default_rng(seed)
    extras = rng.standard_normal((n, extra)).astype(np.float32)
    feats = np.concatenate([colors, extras], axis=1)
    C = feats.shape[1]
    bg = rng.uniform(0.0, 1.0, C).astype(np.float32)
    out.update(colors=colors, extras=extras, background=bg)

    # splatting/binning.py:16-37 with the radial sort distance
    offsets = np.cumsum(tiles, dtype=np.int64).astype(np.int32)
    m = int(offsets[-1]) if n else 0
    keys = np.zeros(2 * m, np.uint64)
    ids = np.zeros(2 * m, np.int32)
    ws.launch(ref["bin"].duplicate, n, [A(centers, wp.vec2), A(radii), A(depths), A(offsets),
                                         gx, gy, A(keys), A(ids)])
    order = np.argsort(keys[:m], kind="stable")
    keys_sorted, ids_sorted = keys[:m][order], ids[:m][order]
    ranges = np.zeros((T, 2), np.int32)
    ws.launch(ref["tiling"].identify_ranges, m, [A(keys_sorted), A(ranges)])
    out.update(keys=keys_sorted, ids=ids_sorted, ranges=ranges)

    # rade/render.py:99-322
    Feature = wp.types.vector(C, np.float32)
    image = np.zeros((C + 6) * H * W, np.float32)
    aux = np.zeros(2 * H * W, np.float32)
    contrib = np.zeros(2 * H * W, np.int32)
    ws.launch(ref["rade_render"]._make_forward(C, ()), 256 * T,
              [W, H, A(ranges), A(ids_sorted), A(centers, wp.vec2), A(conics, wp.vec4),
               A(feats, Feature), A(bg), A(image), A(aux), A(contrib), A(planes, wp.vec3),
               A(normals, wp.vec3), A(K.copy())], block=256)
    out.update(image=image.reshape(C + 6, H, W), auxiliary=aux.reshape(2, H, W),
               contributors=contrib.reshape(2, H, W))

    # rade/render.py:325-547 with every upstream image seeded N(0,1)
    up = {k: rng.standard_normal((H, W, c)).astype(np.float32)
          for k, c in (("up_features", C), ("up_alpha", 1), ("up_depth", 1), ("up_median", 1),
                       ("up_normals", 3))}
    grads = {k: np.zeros((n, c), np.float32)
             for k, c in (("grad_centers", 2), ("grad_conics", 4), ("grad_features", C),
                          ("grad_abs", 2), ("grad_planes", 3), ("grad_normals", 3))}
    ws.launch(ref["rade_render"]._make_backward(C, True), 256 * T,
              [W, H, A(ranges), A(ids_sorted), A(centers, wp.vec2), A(conics, wp.vec4),
               A(feats, Feature), A(bg), A(image), A(aux), A(planes, wp.vec3),
               A(normals, wp.vec3), A(K.copy()), A(contrib),
               *(A(up[k]) for k in ("up_features", "up_alpha", "up_depth", "up_median",
                                    "up_normals")),
               A(grads["grad_centers"], wp.vec2), A(grads["grad_conics"], wp.vec4),
               A(grads["grad_features"], Feature), A(grads["grad_abs"], wp.vec2),
               A(grads["grad_planes"], wp.vec3), A(grads["grad_normals"], wp.vec3)],
              block=256)
    out.update(up)
    out.update(grads)
    print(f"rade_{name}: n={n} visible={int((radii > 0).sum())} pairs={m} tiles={T} C={C} "
          f"kernel_size={kernel_size} in {time.time() - t0:.1f}s", flush=True)
    return out


def rade_scenes(base: dict) -> dict:
    """The c1 geometry (SH3), the dense scene (SH1, early termination, culled
    rows) and its copy with near-degenerate Gaussians: a flat axis below
    1e-7 (rade/projection.py:150-159's outer-product branch) in each of the
    three positions."""
    out = {"c1_sh3": base["c1_sh3"], "dense_sh1": base["dense_sh1"]}
    flat = {k: (v.copy() if isinstance(v, np.ndarray) else v)
            for k, v in base["dense_sh1"].items()}
    for i in range(60, 90):
        flat["scales"][i, i % 3] = 1e-8
    out["flat_sh1"] = flat
    return out


# preprocess_3d's switches, in its argument order (aaa/preprocess3d.py:39-44);
# aaa/preprocess.py:320-321 sets cooperative = load_balancing and tile
# culling, complete = eval_3D and not cooperative.
AAA_FLAGS = ("ewa", "new_aabb", "near_clipping", "tile_culling", "complete", "cooperative")


def aaa_case(name, scene: dict, flags: dict, use_sh: bool, with_filter: bool) -> dict:
    """One view through aaa/preprocess3d.py:17-245 (sort order PTD_MAX = 3, the
    default of aaa/config.py:47)."""
    cams = importlib.import_module("dsl_splat.aaa.cameras")
    pre = importlib.import_module("dsl_splat.aaa.preprocess3d")
    W, H = scene["width"], scene["height"]
    means = scene["means"].astype(np.float32)
    n = len(means)
    quats = F.normalize(torch.from_numpy(scene["quats"].astype(np.float32)), dim=-1).numpy()
    scales = scene["scales"].astype(np.float32)
    opac = scene["opacities"].astype(np.float32)
    deg = scene["sh_degree"] if use_sh else 0
    sh = scene["sh"].astype(np.float32) if use_sh else np.zeros((n, 0, 3), np.float32)
    filters = scene["filters"].astype(np.float32) if with_filter else np.zeros(0, np.float32)
    view = torch.from_numpy(scene["viewmat"].astype(np.float32))
    K = torch.from_numpy(scene["K"].astype(np.float32))
    batch = cams.prepare_cameras(view[None, None], K[None, None], W, H, 0.01, 1e10)
    fx, fy, cx, cy = batch.intrinsics[0][0]
    tanx, tany = W / (2 * fx), H / (2 * fy)
    v = batch.transposed_views[0, 0].numpy().copy()
    proj = batch.projection[0, 0].numpy().copy()
    campos = batch.centers[0, 0].numpy().astype(np.float32).copy()
    wp = sys.modules["warp"]
    centers = np.zeros((n, 2), np.float32)
    rects = np.zeros((n, 2), np.float32)
    depths = np.zeros(n, np.float32)
    transforms = np.zeros((n, 4, 4), np.float32)
    eff = np.zeros(n, np.float32)
    radii = np.zeros(n, np.int32)
    tiles = np.zeros(n, np.int32)
    rgb = np.zeros((n if use_sh else 0, 3), np.float32)
    valid = np.zeros(n, np.bool_)
    clamped = np.zeros((n if use_sh else 0, 3), np.bool_)
    queued = np.full(n, -1, np.int32)
    queue_size = np.zeros(1, np.int32)
    t0 = time.time()
    ws.launch(pre.preprocess_3d, n, [
        A(means, wp.vec3), A(scales, wp.vec3), A(quats, wp.vec4), A(opac),
        A(sh, wp.vec3), use_sh, deg, 3, A(filters), with_filter,
        A(campos[None], wp.vec3), A(v), A(proj), W, H,
        np.float32(tanx), np.float32(tany), np.float32(cx), np.float32(cy), np.float32(1.0),
        *[bool(flags[k]) for k in AAA_FLAGS],
        A(centers, wp.vec2), A(rects, wp.vec2), A(depths), A(transforms, wp.mat44), A(eff),
        A(radii), A(tiles), A(rgb, wp.vec3), A(valid), A(clamped), A(queued), A(queue_size)])
    q = np.sort(queued[:queue_size[0]])
    # aaa/backward_preprocess.py:318-345: focal_x = width / (2 tanfovx) in
    # double, a float32 kernel argument; the raw input opacities
    bwd = importlib.import_module("dsl_splat.aaa.backward_preprocess")
    gen = np.random.default_rng(700 + len(name))
    up_transforms = gen.standard_normal((n, 4, 4)).astype(np.float32)
    up_opacity = gen.standard_normal(n).astype(np.float32)
    focal_x = np.float32(W / (2.0 * tanx))
    adj = dict(opacity=np.zeros(n, np.float32), means=np.zeros((n, 3), np.float32),
               scales=np.zeros((n, 3), np.float32), quats=np.zeros((n, 4), np.float32))
    ws.launch(bwd.preprocess_adjoint, n, [
        A(means, wp.vec3), A(scales, wp.vec3), A(quats, wp.vec4), A(opac), A(radii), A(v),
        A(proj), A(campos[None], wp.vec3), W, H, focal_x, bool(flags["ewa"]),
        A(up_transforms, wp.mat44), A(up_opacity), A(adj["opacity"]), A(adj["means"], wp.vec3),
        A(adj["scales"], wp.vec3), A(adj["quats"], wp.vec4)])
    adjoint = dict(adj_up_transforms=up_transforms, adj_up_opacity=up_opacity,
                   adj_focal_x=focal_x, **{f"adj_{k}": a for k, a in adj.items()})
    # aaa/backward_camera.py:259-290: focal = max of the two focal lengths
    cam_mod = importlib.import_module("dsl_splat.aaa.backward_camera")
    up_colors = gen.standard_normal(n * 3).astype(np.float32)
    focal = np.float32(max(W / (2 * tanx), H / (2 * tany)))
    rows = np.zeros((n, 23), np.float32)
    ws.launch(cam_mod.camera_adjoint, n, [
        A(means, wp.vec3), A(scales, wp.vec3), A(quats, wp.vec4), A(filters), with_filter,
        A(radii), A(eff), A(v), A(proj), A(campos[None], wp.vec3), W, H, focal, np.float32(1.0),
        bool(flags["ewa"]), A(up_transforms, wp.mat44), A(up_opacity), A(sh, wp.vec3), use_sh,
        deg, A(clamped), A(up_colors), A(rows)])
    adjoint.update(cam_up_colors=up_colors, cam_focal=focal, cam_rows=rows)
    final = {}
    if flags["cooperative"]:
        # aaa/preprocess.py:453-476: min(n, 1024) blocks of 32 lanes
        cull = importlib.import_module("dsl_splat.aaa.cooperative_culling")
        f_radii, f_tiles, f_valid = radii.copy(), tiles.copy(), valid.copy()
        ws.launch_tiled(cull.cull_remainder_3d, min(n, 1024), [
            A(centers, wp.vec2), A(rects, wp.vec2), A(transforms, wp.mat44), A(eff), W, H,
            min(n, 1024), A(f_radii), A(f_tiles), A(f_valid), A(queued), A(queue_size)], 32)
        final = dict(final_radii=f_radii, final_tiles=f_tiles, final_valid=f_valid)
        if name == "coop":
            final.update(aaa_duplicate(dict(final, centers=centers, rects=rects,
                                            transforms=transforms, opacity=eff,
                                            width=W, height=H)))
    print(f"aaa_{name}: n={n} visible={int((radii > 0).sum())} queued={len(q)} "
          f"valid={int(valid.sum())} final valid="
          f"{int(final['final_valid'].sum()) if final else '-'} in {time.time() - t0:.1f}s")
    return dict(width=W, height=H, sh_degree=deg, use_sh=use_sh, has_filter=with_filter,
                means=means, quats=quats, scales=scales, opacities=opac, sh=sh,
                filters=filters, view=v, proj=proj, campos=campos,
                tanfov=np.array([tanx, tany], np.float32),
                principal=np.array([cx, cy], np.float32),
                flags=np.array([flags[k] for k in AAA_FLAGS], np.bool_),
                centers=centers, rects=rects, depths=depths, transforms=transforms,
                opacity=eff, radii=radii, tiles=tiles, rgb=rgb, valid=valid,
                clamped=clamped, queued=q, **final, **adjoint)


_DUPLICATE_DRIVER = r"""
static void duplicate_body(int i, wp::array_t<wp::vec_t<2, float>> centers,
                           wp::array_t<wp::vec_t<2, float>> extents, wp::array_t<int> radii,
                           wp::array_t<wp::mat_t<4, 4, float>> transforms,
                           wp::array_t<float> opacity3d, wp::array_t<int> offsets, int width,
                           int height, wp::array_t<uint64_t> keys, wp::array_t<int> values) {
SNIPPET
}
extern "C" void run(int n, float* centers, float* extents, int* radii, float* transforms,
                    float* opacity, int* offsets, int width, int height, uint64_t* keys,
                    int* values, int nkeys) {
  using V2 = wp::vec_t<2, float>;
  using M4 = wp::mat_t<4, 4, float>;
  wp::array_t<V2> c{reinterpret_cast<V2*>(centers), {n}}, e{reinterpret_cast<V2*>(extents), {n}};
  wp::array_t<int> r{radii, {n}}, off{offsets, {n}}, v{values, {nkeys}};
  wp::array_t<M4> t{reinterpret_cast<M4*>(transforms), {n}};
  wp::array_t<float> o{opacity, {n}};
  wp::array_t<uint64_t> k{keys, {nkeys}};
  // aaa/binning_native.py:134-135: threads rounded up to whole warps
  run_warps(((n + 31) / 32) * 32, [&](int i) { duplicate_body(i, c, e, r, t, o, off, width, height, k, v); });
}
"""


def aaa_duplicate(d: dict) -> dict:
    """aaa/binning_native.py:85-135 on a load-balanced case's final rows:
    offsets are the inclusive scan of the visible Gaussians' tile counts."""
    bn = importlib.import_module("dsl_splat.aaa.binning_native")
    snippet = bn._duplicate_cooperative.__wp_snippet__
    lib = ws.compile_warp_snippet(_DUPLICATE_DRIVER.replace("SNIPPET", snippet), "aaa_duplicate")
    radii = d["final_radii"].astype(np.int32)
    offsets = np.cumsum(np.where(radii > 0, d["final_tiles"], 0)).astype(np.int32)
    total = int(offsets[-1])
    keys = np.zeros(total, np.uint64)
    values = np.full(total, -7, np.int32)
    f32 = lambda a: np.ascontiguousarray(a, np.float32)
    centers, rects, transforms, opacity = (f32(d[k]) for k in ("centers", "rects", "transforms",
                                                                "opacity"))
    ptr = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    lib.run.restype = None
    lib.run(ctypes.c_int(len(radii)), ptr(centers), ptr(rects), ptr(radii), ptr(transforms),
            ptr(opacity), ptr(offsets), ctypes.c_int(int(d["width"])),
            ctypes.c_int(int(d["height"])), ptr(keys), ptr(values), ctypes.c_int(total))
    assert (values != -7).all()
    return dict(dup_offsets=offsets, dup_keys=keys, dup_values=values)


def aaa_scenes():
    """Seeded views with small, long (more than 32 tiles, queued) and culled
    Gaussians on a 128x96 image (8x6 tiles)."""
    from dsl_splat_b200.scenes import intrinsics, look_at
    g = torch.Generator().manual_seed(4242)
    n = 320
    means = (torch.rand(n, 3, generator=g) * 2 - 1) * torch.tensor([2.0, 1.5, 1.5])
    means[:, 2] += 5.0
    means[:16, 2] = -1.0 - torch.rand(16, generator=g)          # behind the camera
    means[16:32, 0] += 14.0                                      # off screen
    means[32:40, 2] = 0.05 + 0.1 * torch.rand(8, generator=g)    # near plane
    scales = torch.exp(torch.randn(n, 3, generator=g) * 0.5 - 2.6)
    scales[40:56] = torch.exp(torch.randn(16, 3, generator=g) * 0.3 - 0.2)  # long rects
    scales[56:64] = torch.tensor([1e-4, 1e-4, 1e-4])             # sub-pixel
    opac = torch.sigmoid(torch.randn(n, generator=g) + 1.0)
    opac[64:72] = 0.002                                          # below 1/255
    sh = torch.empty(n, 16, 3)
    sh[:, 0] = torch.rand(n, 3, generator=g) * 2 - 0.5
    sh[:, 1:] = torch.randn(n, 15, 3, generator=g) * 0.2
    base = dict(width=128, height=96, sh_degree=3, means=means.numpy(), scales=scales.numpy(),
                quats=torch.randn(n, 4, generator=g).numpy(), opacities=opac.numpy(),
                sh=sh.numpy(), filters=(torch.rand(n, generator=g) * 0.02).numpy(),
                viewmat=look_at(torch.tensor([0.6, -0.4, -1.0]),
                                torch.tensor([0.0, 0.0, 5.0])).numpy(),
                K=intrinsics(110.0, 104.0, 63.0, 49.5).numpy())
    coop = dict(ewa=True, new_aabb=True, near_clipping=False, tile_culling=True,
                complete=False, cooperative=True)
    return [
        ("coop", base, coop, False, False),                       # aaa.rasterize defaults
        ("coop_sh3_filter", base, coop, True, True),
        ("complete", base, dict(coop, complete=True, cooperative=False), True, False),
        ("screen_bounds", base, dict(coop, ewa=False, new_aabb=False, near_clipping=True,
                                     complete=True, cooperative=False), False, True),
        ("noculling", base, dict(coop, tile_culling=False, cooperative=False), False, False),
    ]


def aaa_render_case(name, scene: dict, channels: int, cull: bool, seed: int,
                    statistics: bool = False) -> dict:
    """The AAA HIER 64/8/4 blend and its replay backward, the reference's own
    Warp kernels, on one view of the load-balanced path:
      aaa/preprocess3d.py:17-245 + aaa/cooperative_culling.py:152-192 +
      aaa/binning_native.py:7-135 (through aaa_case / aaa_duplicate),
      the 64-bit key sort restated (stable, end_bit = 32 + bit_length(T)),
      primitives/tiling.py:39-54              identify_ranges,
      aaa/render_hierarchical_warp.py:599-691 render (C channels),
      aaa/backward_render.py:75-137           replay (screen and absgrad
                                              statistics on).
    Features are seeded U[0,1] with a constant last channel (aaa/api.py:
    67-71 appends ones), the background seeded U[0,1] (0 for the constant
    channel), the upstream image gradient seeded N(0,1).  With statistics the
    forward is the reference's render_statistics kernel (:608-653, the
    observer of statistics.py:47-73 in blend_step) with a masked count over
    the upper half and a weighted sum of seeded U[0,1] pixel weights."""
    flags = dict(ewa=True, new_aabb=True, near_clipping=False, tile_culling=True,
                 complete=False, cooperative=True)
    pre = aaa_case("coop", scene, flags, False, False)
    W, H = int(pre["width"]), int(pre["height"])
    gx, gy = (W + 15) // 16, (H + 15) // 16
    T = gx * gy
    keys, values = pre["dup_keys"], pre["dup_values"]
    end_bit = 32 + T.bit_length()
    order = np.argsort(keys & np.uint64((1 << end_bit) - 1), kind="stable")
    skeys, ids = keys[order], values[order].astype(np.int32)
    tiling = importlib.import_module("dsl_splat.primitives.tiling")
    ranges = np.zeros((T, 2), np.int32)
    wp = sys.modules["warp"]
    if len(skeys):
        ws.launch(tiling.identify_ranges, len(skeys), [A(skeys), A(ranges)])
    n = len(pre["means"])
    gen = np.random.default_rng(seed)
    feats = gen.uniform(0, 1, (n, channels)).astype(np.float32)
    feats[:, -1] = 1.0
    bg = gen.uniform(0, 1, channels).astype(np.float32)
    bg[-1] = 0.0
    warp_render = importlib.import_module("dsl_splat.aaa.render_hierarchical_warp")
    backward = importlib.import_module("dsl_splat.aaa.backward_render")
    ftype = wp.types.vector(channels, wp.float32)
    image = np.zeros(channels * H * W, np.float32)
    final_t = np.zeros(H * W, np.float32)
    contrib = np.zeros(H * W, np.int32)
    transforms = pre["transforms"].astype(np.float32)
    opacity = pre["opacity"].astype(np.float32)
    t0 = time.time()
    stats = {}
    args = [W, H, A(ranges.reshape(-1)), A(ids), A(transforms, wp.mat44), A(opacity),
            A(feats, ftype), A(bg), A(image), A(final_t), A(contrib)]
    if statistics:
        mask = np.zeros((H, W), np.float32)
        mask[: H // 2] = 1.0
        weights = gen.uniform(0.0, 1.0, (H, W)).astype(np.float32)
        pixel_values = np.stack([mask.ravel(), weights.ravel()])  # request 0 count, 1 sum
        counts = np.zeros((1, n), np.int32)
        sums = np.zeros((1, n), np.float32)
        kernel = warp_render._make_kernel(cull, channels, (0, 1))
        args += [A(pixel_values), A(counts), A(sums)]
        stats = dict(stat_mask=mask, stat_weights=weights, stat_counts=counts[0],
                     stat_sums=sums[0])
    else:
        kernel = warp_render._make_kernel(cull, channels)
    ws.launch(kernel, 256 * T, args, block=256)
    t1 = time.time()
    up = gen.standard_normal(channels * H * W).astype(np.float32)
    g_tr = np.zeros(n * 16, np.float32)
    g_op = np.zeros(n, np.float32)
    g_col = np.zeros(n * channels, np.float32)
    g_scr = np.zeros(n * 2, np.float32)
    g_abs = np.zeros(n * 2, np.float32)
    replay = backward._make_backward(cull, channels, True, True)
    ws.launch(replay, 256 * T, [W, H, A(ranges.reshape(-1)), A(ids), A(feats, ftype), A(image),
                                A(final_t), A(contrib), A(transforms, wp.mat44), A(opacity),
                                A(bg), A(up), A(g_tr), A(g_op), A(g_col), A(g_scr), A(g_abs)],
              block=256)
    print(f"aaa_render_{name}: {W}x{H} C={channels} cull={cull} pairs={len(ids)} "
          f"max contributors={contrib.max()} forward {t1 - t0:.1f}s "
          f"backward {time.time() - t1:.1f}s")
    return dict(width=W, height=H, channels=channels, cull=cull, ranges=ranges, ids=ids,
                transforms=transforms, opacity=opacity, features=feats, background=bg,
                image=image.reshape(channels, H, W), final_t=final_t.reshape(H, W),
                contributors=contrib.reshape(H, W), upstream=up.reshape(channels, H, W),
                grad_transforms=g_tr.reshape(n, 16), grad_opacity=g_op,
                grad_features=g_col.reshape(n, channels), grad_screen=g_scr.reshape(n, 2),
                grad_screen_abs=g_abs.reshape(n, 2), **stats)


def aaa_render_scenes():
    """Render cases: the sparse preprocessing scene, and a dense one (700
    Gaussians on a 44x36 image, ragged tiles) whose 4x4 tails overflow, so
    every queue path (tail drains, mid merges, full heads, early
    termination) runs."""
    from dsl_splat_b200.scenes import intrinsics, look_at
    base = aaa_scenes()[0][1]
    g = torch.Generator().manual_seed(777)
    n = 700
    means = (torch.rand(n, 3, generator=g) * 2 - 1) * torch.tensor([1.2, 1.0, 0.8])
    means[:, 2] += 4.0
    scales = torch.exp(torch.randn(n, 3, generator=g) * 0.4 - 2.0)
    opac = torch.sigmoid(torch.randn(n, generator=g) + 0.5)
    dense = dict(width=44, height=36, sh_degree=3, means=means.numpy(), scales=scales.numpy(),
                 quats=torch.randn(n, 4, generator=g).numpy(), opacities=opac.numpy(),
                 sh=np.zeros((n, 16, 3), np.float32), filters=np.zeros(n, np.float32),
                 viewmat=look_at(torch.tensor([0.2, -0.1, -1.0]),
                                 torch.tensor([0.0, 0.0, 4.0])).numpy(),
                 K=intrinsics(40.0, 38.0, 21.5, 17.5).numpy())
    return [("sparse_c4", base, 4, True, 11, False), ("dense_c7", dense, 7, True, 12, True),
            ("dense_nocull_c4", dense, 4, False, 13, False)]


def tile_mode_case(ref, name, scene: dict) -> dict:
    """Projection tile counts and binning for tile_mode snugbox and accutile
    (gs3d/projection.py:150-162, splatting/intersections.py:45-218,
    splatting/binning.py:40-117): the reference's own kernels."""
    W, H = scene["width"], scene["height"]
    gx, gy = (W + 15) // 16, (H + 15) // 16
    T = gx * gy
    means = scene["means"].astype(np.float32)
    n = len(means)
    quats = F.normalize(torch.from_numpy(scene["quats"].astype(np.float32)), dim=-1).numpy()
    scales = scene["scales"].astype(np.float32)
    opac = scene["opacities"].astype(np.float32)
    view = scene["viewmat"].astype(np.float32)
    K = scene["K"].astype(np.float32)
    wp = sys.modules["warp"]
    full = np.zeros((1, 4, 4), np.float32)
    inverse = np.zeros((1, 4, 4), np.float32)
    centers_cam = np.zeros((1, 3), np.float32)
    errors = np.zeros(1, np.int32)
    ws.launch(ref["cam"].prepare_kernel, 1,
              [A(view[None].copy()), A(K[None].copy()), W, H, 1, A(full), A(inverse),
               A(centers_cam), A(errors)])
    out: dict = dict(width=W, height=H, means=means, quats=quats, scales=scales,
                     opacities=opac, viewmat=view, K=K, full=full[0])
    t0 = time.time()
    for mode in ("snugbox", "accutile"):
        centers = np.zeros((n, 2), np.float32)
        conics = np.zeros((n, 4), np.float32)
        radii = np.zeros(n, np.int32)
        tiles = np.zeros(n, np.int32)
        depths = np.zeros(n, np.float32)
        ws.launch(ref["proj"]._make_project(mode), n,
                  [A(means, wp.vec3), A(quats, wp.vec4), A(scales, wp.vec3), A(opac),
                   A(view.copy()), A(full[0].copy()), A(K.copy()), W, H, np.float32(0.2),
                   np.float32(np.inf), np.float32(0.0), A(centers, wp.vec2),
                   A(conics, wp.vec4), A(radii), A(tiles), A(depths)])
        offsets = np.cumsum(tiles, dtype=np.int64).astype(np.int32)
        m = int(offsets[-1]) if n else 0
        keys = np.zeros(2 * m, np.uint64)
        ids = np.zeros(2 * m, np.int32)
        ws.launch(ref["bin"]._make_duplicate(mode), n,
                  [A(centers, wp.vec2), A(conics, wp.vec4), A(radii), A(depths), A(offsets),
                   gx, gy, A(keys), A(ids)])
        order = np.argsort(keys[:m], kind="stable")
        ranges = np.zeros((T, 2), np.int32)
        ws.launch(ref["tiling"].identify_ranges, m, [A(keys[:m][order]), A(ranges)])
        out.update({f"{mode}_centers": centers, f"{mode}_conics": conics,
                    f"{mode}_radii": radii, f"{mode}_tiles": tiles, f"{mode}_depths": depths,
                    f"{mode}_keys": keys[:m][order], f"{mode}_ids": ids[:m][order],
                    f"{mode}_ranges": ranges})
        print(f"{name} {mode}: visible={int((radii > 0).sum())} pairs={m}", flush=True)
    print(f"{name}: {time.time() - t0:.1f}s", flush=True)
    return out


def tile_mode_scenes(base: dict) -> dict:
    """The c1/dense geometries plus an edge scene: thin rotated ellipses,
    opacities on both sides of 1/255 and footprints larger than the image."""
    from dsl_splat_b200.scenes import intrinsics
    out = {k: base[k] for k in ("c1_sh3", "dense_sh1")}
    g = torch.Generator().manual_seed(77)
    n = 300
    means = (torch.rand(n, 3, generator=g) * 2 - 1) * torch.tensor([1.6, 1.2, 0.0])
    means[:, 2] = 3.0 + torch.rand(n, generator=g) * 3
    scales = torch.exp(torch.randn(n, 3, generator=g) * 0.8 - 2.5)
    scales[:100, 0] *= 20.0                       # long along x
    scales[100:150, 1] *= 30.0                    # long along y
    scales[150:160] = torch.tensor([2.5, 2.5, 2.5])  # larger than the image
    opac = torch.sigmoid(torch.randn(n, generator=g) * 3)
    opac[160:180] = 1.0 / 255.0 * (0.5 + torch.rand(20, generator=g))  # around the threshold
    opac[180:185] = 1.0
    out["edges"] = dict(width=72, height=56, means=means.numpy(), scales=scales.numpy(),
                        quats=torch.randn(n, 4, generator=g).numpy(), opacities=opac.numpy(),
                        viewmat=torch.eye(4).numpy(), K=intrinsics(60.0, 60.0, 36.0, 28.0).numpy())
    return out


def scenes():
    """Small seeded scenes with the benchmark configs' distributions."""
    from dsl_splat_b200.scenes import intrinsics, look_at
    g = torch.Generator().manual_seed(2024)
    out = {}
    # config-0 shapes: box in front of an identity camera, SH0
    n = 160
    xy = torch.rand(n, 2, generator=g) * 2 - 1
    z = torch.rand(n, 1, generator=g) * 4 + 2
    out["c0_sh0"] = dict(
        width=48, height=40, sh_degree=0, means=torch.cat([xy, z], 1).numpy(),
        scales=torch.exp(torch.randn(n, 3, generator=g) * 0.5 - 3.0).numpy(),
        quats=torch.randn(n, 4, generator=g).numpy(),
        opacities=torch.sigmoid(torch.randn(n, generator=g)).numpy(),
        sh=torch.rand(n, 1, 3, generator=g).numpy(),
        viewmat=torch.eye(4).numpy(), K=intrinsics(48.0, 48.0, 24.0, 20.0).numpy())
    # config-1 shapes: clustered ball, SH3, camera at distance 8, rotated view
    n = 220
    centres = (torch.rand(8, 3, generator=g) * 2 - 1) * 3
    means = centres[torch.randint(0, 8, (n,), generator=g)] + 0.5 * torch.randn(n, 3, generator=g)
    sh = torch.empty(n, 16, 3)
    sh[:, 0] = torch.rand(n, 3, generator=g)
    sh[:, 1:] = torch.randn(n, 15, 3, generator=g) * 0.1
    out["c1_sh3"] = dict(
        width=56, height=40, sh_degree=3, means=means.numpy(),
        scales=torch.exp(torch.randn(n, 3, generator=g) * 0.7 - 2.0).numpy(),
        quats=torch.randn(n, 4, generator=g).numpy(),
        opacities=torch.sigmoid(torch.randn(n, generator=g)).numpy(),
        sh=sh.numpy(),
        viewmat=look_at(torch.tensor([2.0, -1.0, -8.0])).numpy(),
        K=intrinsics(60.0, 60.0, 28.0, 20.0).numpy())
    # dense overlap (early termination), Gaussians behind the camera, off
    # screen and one covering every tile; SH1, off-centre principal point
    n = 420
    means = (torch.rand(n, 3, generator=g) * 2 - 1) * torch.tensor([1.5, 1.2, 1.0])
    means[:, 2] += 4.0
    means[:20, 2] = -1.0 - torch.rand(20, generator=g)        # behind the camera
    means[20:40, 0] += 12.0                                    # far off screen
    means[40] = torch.tensor([0.0, 0.0, 3.0])
    scales = torch.exp(torch.randn(n, 3, generator=g) * 0.4 - 2.3)
    scales[40] = torch.tensor([1.5, 1.5, 1.5])                 # spans every tile
    opac = torch.sigmoid(torch.randn(n, generator=g) + 2.0)
    sh = torch.empty(n, 4, 3)
    sh[:, 0] = torch.rand(n, 3, generator=g)
    sh[:, 1:] = torch.randn(n, 3, 3, generator=g) * 0.2
    out["dense_sh1"] = dict(
        width=64, height=48, sh_degree=1, means=means.numpy(), scales=scales.numpy(),
        quats=torch.randn(n, 4, generator=g).numpy(), opacities=opac.numpy(), sh=sh.numpy(),
        viewmat=look_at(torch.tensor([0.5, -0.3, -1.0]), torch.tensor([0.0, 0.0, 4.0])).numpy(),
        K=intrinsics(56.0, 52.0, 30.5, 25.0).numpy())
    return out


def main():
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    ref_root = args[0] if args else os.environ.get("DSL_SPLAT_REFERENCE")
    if not ref_root:
        raise SystemExit("usage: make_golden.py <dsl_splat checkout> [--...-only] "
                         "(or set DSL_SPLAT_REFERENCE)")
    ref = load_reference(ref_root)
    base = scenes()
    only = {a for a in sys.argv[1:]
            if a in ("--tile-modes-only", "--wide-only", "--rade-only", "--aaa-only",
                     "--aaa-render-only")}
    if not only:
        for i, (name, scene) in enumerate(base.items()):
            data = golden_case(ref, name, scene, seed=100 + i)
            np.savez_compressed(os.path.join(HERE, f"gs3d_{name}.npz"), **data)
    if not only or "--wide-only" in only:
        for name in ("c1_sh3", "dense_sh1"):
            data = wide_case(ref, name, base[name], seed=300)
            np.savez_compressed(os.path.join(HERE, f"wide_{name}.npz"), **data)
    if not only or "--rade-only" in only:
        for name, ks, extra in (("c1_sh3", 0.0, 4), ("dense_sh1", 0.3, 0), ("flat_sh1", 0.1, 5)):
            data = rade_case(ref, name, rade_scenes(base)[name], 500, ks, extra)
            np.savez_compressed(os.path.join(HERE, f"rade_{name}.npz"), **data)
    if not only or "--aaa-only" in only:
        for name, scene, flags, use_sh, with_filter in aaa_scenes():
            data = aaa_case(name, scene, flags, use_sh, with_filter)
            np.savez_compressed(os.path.join(HERE, f"aaa_{name}.npz"), **data)
    if not only or "--aaa-render-only" in only:
        for name, scene, channels, cull, seed, statistics in aaa_render_scenes():
            data = aaa_render_case(name, scene, channels, cull, seed, statistics)
            np.savez_compressed(os.path.join(HERE, f"aaa_render_{name}.npz"), **data)
    if only and "--tile-modes-only" not in only:
        return
    for name, scene in tile_mode_scenes(base).items():
        data = tile_mode_case(ref, name, scene)
        np.savez_compressed(os.path.join(HERE, f"tilemodes_{name}.npz"), **data)


if __name__ == "__main__":
    main()
