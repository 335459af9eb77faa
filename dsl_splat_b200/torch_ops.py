"""torch.ops.splat200.*: the C-ABI stages as schema'd PyTorch operators.

Each operator is the matching `stages` call (one launch sequence through
libsplat200.so on the current stream) registered with torch.library, with a
fake implementation that gives output shapes and dtypes without running the
kernels -- so the stages trace under FakeTensorMode, torch.compile and
torch.export.  The differentiable ones (`project`, `sh_forward`, `render`)
carry autograd formulas that call the backward operators, so a graph built
from them stays inside torch.ops.splat200.

Binning's pair count is data-dependent: its fake kernel returns an unbacked
size for point_list, which is what the reference's `.item()` read
(primitives/tiling.py:64) becomes in a traced graph.

Operator <- reference code it stands for:
  cameras_prepare     splatting/cameras.py:29-85 (camera_kernels.py:11-66)
  project             gs3d/projection.py:309-354 (tile counts for tile_mode)
  project_backward    gs3d/projection.py:357-428
  project_views       gs3d/api.py:132-189 (the per-camera projection loop, one launch)
  project_views_backward  the per-camera backward calls of that loop, summed
  sh_forward          primitives/spherical_harmonics.py:18-59 (sh.py:44-79)
  sh_backward         primitives/spherical_harmonics.py:61-101 (sh.py:82-138)
  bin_and_sort        splatting/binning.py:72-117
  render              gs3d/render.py:359-406 (features + a constant alpha channel)
  render_backward     gs3d/render.py:409-463
  rade_project        rade/projection.py:422-472 (ray planes, normals, radial depths)
  rade_project_backward  rade/projection.py:475-551
  rade_render         rade/render.py:550-601 (colour, alpha, depths, normals)
  rade_render_backward   rade/render.py:604-670
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import stages

_NS = "splat200"


def _state(centers, conics, radii, tiles, depths) -> stages.ProjectedGaussians:
    return stages.ProjectedGaussians(centers, conics, radii, tiles, depths)


# ---- cameras -------------------------------------------------------------------

@torch.library.custom_op(f"{_NS}::cameras_prepare", mutates_args=())
def cameras_prepare(views: Tensor, Ks: Tensor, width: int, height: int,
                    with_centers: bool) -> tuple[Tensor, Tensor, Tensor]:
    full, inverse, centers = stages.cameras_prepare(views, Ks, width, height, with_centers)
    return full, inverse, centers


@cameras_prepare.register_fake
def _(views, Ks, width, height, with_centers):
    count = views.numel() // 16
    full = views.new_empty(views.shape)
    inverse = views.new_empty((count if with_centers else 0, 4, 4))
    centers = views.new_empty(views.shape[:-2] + (3,) if with_centers else (0, 3))
    return full, inverse, centers


# ---- projection ----------------------------------------------------------------

@torch.library.custom_op(f"{_NS}::project", mutates_args=())
def project(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor, view: Tensor,
            full: Tensor, K: Tensor, width: int, height: int, near: float, far: float,
            radius_clip: float, tile_mode: str) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    st = stages.project(means, quats, scales, opacities, view, full, K, width, height, near,
                        far, radius_clip, tile_mode)
    return st.centers, st.conics, st.radii, st.tile_counts, st.depths


@project.register_fake
def _(means, quats, scales, opacities, view, full, K, width, height, near, far, radius_clip,
      tile_mode):
    n = means.shape[0]
    return (means.new_empty((n, 2)), means.new_empty((n, 4)),
            means.new_empty((n,), dtype=torch.int32), means.new_empty((n,), dtype=torch.int32),
            means.new_empty((n,)))


@torch.library.custom_op(f"{_NS}::project_backward", mutates_args=())
def project_backward(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor,
                     view: Tensor, full: Tensor, K: Tensor, width: int, height: int,
                     centers: Tensor, conics: Tensor, radii: Tensor, tiles: Tensor,
                     depths: Tensor, grad_centers: Tensor, grad_conics: Tensor
                     ) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    grads = stages.project_backward(means, quats, scales, opacities, view, full, K, width, height,
                                    _state(centers, conics, radii, tiles, depths),
                                    grad_centers.contiguous(), grad_conics.contiguous(),
                                    (True,) * 6)
    # the two 4x4 camera gradients are views of one buffer: operator outputs
    # must not alias each other
    return tuple(g.clone() if i >= 4 else g for i, g in enumerate(grads))


@project_backward.register_fake
def _(means, quats, scales, opacities, view, full, K, width, height, centers, conics, radii,
      tiles, depths, grad_centers, grad_conics):
    return (torch.empty_like(means), torch.empty_like(quats), torch.empty_like(scales),
            torch.empty_like(opacities), view.new_empty((4, 4)), full.new_empty((4, 4)))


def _project_setup(ctx, inputs, output):
    means, quats, scales, opacities, view, full, K, width, height, *_ = inputs
    ctx.save_for_backward(means, quats, scales, opacities, view, full, K, *output)
    ctx.size = (width, height)


def _project_backward(ctx, g_centers, g_conics, g_radii, g_tiles, g_depths):
    means, quats, scales, opacities, view, full, K, centers, conics, radii, tiles, depths = \
        ctx.saved_tensors
    g_centers = torch.zeros_like(centers) if g_centers is None else g_centers
    g_conics = torch.zeros_like(conics) if g_conics is None else g_conics
    grads = torch.ops.splat200.project_backward(means, quats, scales, opacities, view, full, K,
                                                *ctx.size, centers, conics, radii, tiles, depths,
                                                g_centers, g_conics)
    return (*grads, None, None, None, None, None, None, None)


project.register_autograd(_project_backward, setup_context=_project_setup)


@torch.library.custom_op(f"{_NS}::project_views", mutates_args=())
def project_views(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor,
                  views: Tensor, fulls: Tensor, Ks: Tensor, width: int, height: int, near: float,
                  far: float, radius_clip: float, sh: Tensor, sh_degree: int, campos: Tensor,
                  tile_mode: str) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """All cameras (V) of one Gaussian set in one launch (raw quaternions are
    normalised in-kernel).  Returns stacked (V, n, ...) centres, conics,
    colours, radii, tile counts, depths and the active mask."""
    out = stages.project_views(means, quats, scales, opacities, views, fulls, Ks, width, height,
                               near, far, radius_clip, sh=sh, sh_degree=sh_degree,
                               campos=campos, normalize_quats=True, tile_mode=tile_mode)
    return (torch.stack(out.centers), torch.stack(out.conics), torch.stack(out.colors),
            out.radii, out.tile_counts, out.depths, out.active)


@project_views.register_fake
def _(means, quats, scales, opacities, views, fulls, Ks, width, height, near, far, radius_clip,
      sh, sh_degree, campos, tile_mode):
    V, n = views.shape[0], means.shape[0]
    return (means.new_empty((V, n, 2)), means.new_empty((V, n, 4)), means.new_empty((V, n, 3)),
            means.new_empty((V, n), dtype=torch.int32), means.new_empty((V, n), dtype=torch.int32),
            means.new_empty((V, n)), means.new_empty((V, n, 3), dtype=torch.uint8))


@torch.library.custom_op(f"{_NS}::project_views_backward", mutates_args=())
def project_views_backward(means: Tensor, quats: Tensor, scales: Tensor, views: Tensor,
                           fulls: Tensor, Ks: Tensor, width: int, height: int, radii: Tensor,
                           sh: Tensor, sh_degree: int, campos: Tensor, active: Tensor,
                           grad_centers: Tensor, grad_conics: Tensor, grad_colors: Tensor
                           ) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Gradients of means, raw quaternions, scales, opacities and SH summed
    over the V cameras (splat_project_backward_views)."""
    V, n = views.shape[0], means.shape[0]
    outs = [torch.empty_like(t) for t in (means, quats, scales)]
    outs.append(means.new_empty(n))
    outs.append(torch.empty_like(sh))
    gc, gq, gcol = grad_centers.contiguous(), grad_conics.contiguous(), grad_colors.contiguous()
    if n and V:
        pin = stages.Args()
        from ._native import check, lib, stream
        check(lib.splat_project_backward_views(
            V, n, pin(means), None, pin(quats), pin(scales), pin(views), pin(fulls), pin(Ks),
            width, height, stages.pointer_table(radii), stages.pointer_table(gc),
            stages.pointer_table(gq), *[o.data_ptr() for o in outs[:4]], 0, sh_degree,
            sh.shape[1], pin(sh), pin(campos), stages.pointer_table(active),
            stages.pointer_table(gcol), 3, outs[4].data_ptr(), stream(means.device)),
            "project_views_backward")
    return tuple(outs)


@project_views_backward.register_fake
def _(means, quats, scales, views, fulls, Ks, width, height, radii, sh, sh_degree, campos,
      active, grad_centers, grad_conics, grad_colors):
    return (torch.empty_like(means), torch.empty_like(quats), torch.empty_like(scales),
            means.new_empty(means.shape[0]), torch.empty_like(sh))


def _project_views_setup(ctx, inputs, output):
    (means, quats, scales, opacities, views, fulls, Ks, width, height, near, far, radius_clip,
     sh, sh_degree, campos, tile_mode) = inputs
    ctx.save_for_backward(means, quats, scales, views, fulls, Ks, sh, campos, output[3],
                          output[6])
    ctx.args = (width, height, sh_degree)


def _project_views_backward(ctx, g_centers, g_conics, g_colors, *unused):
    means, quats, scales, views, fulls, Ks, sh, campos, radii, active = ctx.saved_tensors
    width, height, sh_degree = ctx.args
    V, n = views.shape[0], means.shape[0]

    def zeros(g, k):
        return means.new_zeros((V, n, k)) if g is None else g

    grads = torch.ops.splat200.project_views_backward(
        means, quats, scales, views, fulls, Ks, width, height, radii, sh, sh_degree, campos,
        active, zeros(g_centers, 2), zeros(g_conics, 4), zeros(g_colors, 3))
    gm, gq, gs, go, gsh = grads
    return (gm, gq, gs, go, None, None, None, None, None, None, None, None, gsh, None, None,
            None)


project_views.register_autograd(_project_views_backward, setup_context=_project_views_setup)


# ---- spherical harmonics ------------------------------------------------------------

@torch.library.custom_op(f"{_NS}::sh_forward", mutates_args=())
def sh_forward(coeffs: Tensor, dirs: Tensor, degree: int,
               radii: Tensor | None) -> tuple[Tensor, Tensor]:
    colors, active = stages.sh_forward(coeffs, dirs, degree, radii, True)
    return colors, active


@sh_forward.register_fake
def _(coeffs, dirs, degree, radii):
    n = coeffs.shape[0]
    return coeffs.new_empty((n, 3)), coeffs.new_empty((n, 3), dtype=torch.uint8)


@torch.library.custom_op(f"{_NS}::sh_backward", mutates_args=())
def sh_backward(coeffs: Tensor, dirs: Tensor, degree: int, radii: Tensor | None,
                active: Tensor, grad_colors: Tensor) -> tuple[Tensor, Tensor]:
    g_coeffs, g_dirs = stages.sh_backward(coeffs, dirs, degree, radii, active,
                                          grad_colors.contiguous(), True)
    return g_coeffs, g_dirs


@sh_backward.register_fake
def _(coeffs, dirs, degree, radii, active, grad_colors):
    return torch.empty_like(coeffs), dirs.new_empty((dirs.shape[0], 3))


def _sh_setup(ctx, inputs, output):
    coeffs, dirs, degree, radii = inputs
    ctx.save_for_backward(coeffs, dirs, radii, output[1])
    ctx.degree = degree


def _sh_backward(ctx, g_colors, g_active):
    coeffs, dirs, radii, active = ctx.saved_tensors
    if g_colors is None:
        return None, None, None, None
    g_coeffs, g_dirs = torch.ops.splat200.sh_backward(coeffs, dirs, ctx.degree, radii, active,
                                                      g_colors)
    return g_coeffs, g_dirs, None, None


sh_forward.register_autograd(_sh_backward, setup_context=_sh_setup)


# ---- binning -----------------------------------------------------------------------

@torch.library.custom_op(f"{_NS}::bin_and_sort", mutates_args=())
def bin_and_sort(centers: Tensor, conics: Tensor, radii: Tensor, tiles: Tensor, depths: Tensor,
                 width: int, height: int, tile_mode: str) -> tuple[Tensor, Tensor]:
    bins = stages.bin_and_sort(_state(centers, conics, radii, tiles, depths), width, height,
                               tile_mode=tile_mode)
    return bins["ranges"], bins["point_list"]


@bin_and_sort.register_fake
def _(centers, conics, radii, tiles, depths, width, height, tile_mode):
    T = ((width + 15) // 16) * ((height + 15) // 16)
    pairs = torch.library.get_ctx().new_dynamic_size()
    return (radii.new_empty((T, 2), dtype=torch.int32),
            radii.new_empty((pairs,), dtype=torch.int32))


# ---- blending ----------------------------------------------------------------------

@torch.library.custom_op(f"{_NS}::render", mutates_args=())
def render(centers: Tensor, conics: Tensor, ranges: Tensor, point_list: Tensor,
           features: Tensor, background: Tensor, width: int,
           height: int) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """features (N, C) blended with a constant alpha channel; background (C+1).
    Returns image (H, W, C), alpha (H, W, 1), transmittance (H, W) and
    contributor counts (H, W)."""
    out = stages.render(stages.ProjectedFootprint(centers, conics),
                        dict(ranges=ranges, point_list=point_list), features, None, True,
                        background, width, height, separate_alpha=True)
    return out.features, out.alpha, out.transmittance, out.contributors


@render.register_fake
def _(centers, conics, ranges, point_list, features, background, width, height):
    C = features.shape[1]
    return (features.new_empty((height, width, C)), features.new_empty((height, width, 1)),
            features.new_empty((height, width)),
            features.new_empty((height, width), dtype=torch.int32))


@torch.library.custom_op(f"{_NS}::render_backward", mutates_args=())
def render_backward(centers: Tensor, conics: Tensor, ranges: Tensor, point_list: Tensor,
                    features: Tensor, background: Tensor, transmittance: Tensor,
                    contributors: Tensor, grad_image: Tensor, grad_alpha: Tensor, width: int,
                    height: int) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """Gradients of centers, conics, features and the |d centers| sums."""
    gc, gq, gf, _, gabs = stages.render_backward(
        stages.ProjectedFootprint(centers, conics), dict(ranges=ranges, point_list=point_list),
        features, None, True, background, transmittance, contributors, grad_image, width,
        height, absgrad=True, constant_tail=1, gradient_alpha=grad_alpha, separate_alpha=True,
        separate_buffers=True)
    return gc, gq, gf, gabs


@render_backward.register_fake
def _(centers, conics, ranges, point_list, features, background, transmittance, contributors,
      grad_image, grad_alpha, width, height):
    return (torch.empty_like(centers), torch.empty_like(conics), torch.empty_like(features),
            torch.empty_like(centers))


def _render_setup(ctx, inputs, output):
    centers, conics, ranges, point_list, features, background, width, height = inputs
    ctx.save_for_backward(centers, conics, ranges, point_list, features, background, output[2],
                          output[3])
    ctx.size = (width, height)


def _render_backward(ctx, g_image, g_alpha, g_t, g_contrib):
    centers, conics, ranges, point_list, features, background, final_t, contrib = \
        ctx.saved_tensors
    W, H = ctx.size
    if g_image is None:
        g_image = features.new_zeros((H, W, features.shape[1]))
    if g_alpha is None:
        g_alpha = features.new_zeros((H, W, 1))
    gc, gq, gf, _ = torch.ops.splat200.render_backward(
        centers, conics, ranges, point_list, features, background, final_t, contrib,
        g_image.contiguous(), g_alpha.contiguous(), W, H)
    return gc, gq, None, None, gf, None, None, None


render.register_autograd(_render_backward, setup_context=_render_setup)

# ---- RaDe-GS -----------------------------------------------------------------------

def _rade_config(width, height, near, far, radius_clip, kernel_size):
    from .rade.projection import ViewConfig
    return ViewConfig(width, height, near, far, radius_clip, "radius", kernel_size)


@torch.library.custom_op(f"{_NS}::rade_project", mutates_args=())
def rade_project(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor, view: Tensor,
                 full: Tensor, K: Tensor, width: int, height: int, near: float, far: float,
                 radius_clip: float, kernel_size: float
                 ) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Normalised quats.  Returns centers, conics, radii, tile counts, radial
    sort distances, ray planes and normals."""
    from .rade import projection as rp
    st = rp.prepare(means, quats, scales, opacities, view, full, K,
                    _rade_config(width, height, near, far, radius_clip, kernel_size))
    return (st.centers, st.conics, st.radii, st.tile_counts, st.depths, st.ray_planes,
            st.normals)


@rade_project.register_fake
def _(means, quats, scales, opacities, view, full, K, width, height, near, far, radius_clip,
      kernel_size):
    n = means.shape[0]
    i32 = dict(dtype=torch.int32)
    return (means.new_empty((n, 2)), means.new_empty((n, 4)), means.new_empty((n,), **i32),
            means.new_empty((n,), **i32), means.new_empty((n,)), means.new_empty((n, 3)),
            means.new_empty((n, 3)))


@torch.library.custom_op(f"{_NS}::rade_project_backward", mutates_args=())
def rade_project_backward(means: Tensor, quats: Tensor, scales: Tensor, opacities: Tensor,
                          view: Tensor, full: Tensor, K: Tensor, width: int, height: int,
                          kernel_size: float, radii: Tensor, grad_centers: Tensor,
                          grad_conics: Tensor, grad_planes: Tensor, grad_normals: Tensor
                          ) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    from .rade import projection as rp
    cfg = _rade_config(width, height, 0.0, 0.0, 0.0, kernel_size)
    state = rp.ProjectedGaussians(None, None, radii, None, None, None, None)
    grads = rp.backward(means, quats, scales, opacities, view, full, K, cfg, state,
                        grad_centers.contiguous(), grad_conics.contiguous(),
                        grad_planes.contiguous(), grad_normals.contiguous(), (True,) * 6)
    # the two 4x4 camera gradients are views of one buffer: operator outputs
    # must not alias each other
    return tuple(g.clone() if i >= 4 else g for i, g in enumerate(grads[:6]))


@rade_project_backward.register_fake
def _(means, quats, scales, opacities, view, full, K, width, height, kernel_size, radii,
      grad_centers, grad_conics, grad_planes, grad_normals):
    return (torch.empty_like(means), torch.empty_like(quats), torch.empty_like(scales),
            torch.empty_like(opacities), view.new_empty((4, 4)), full.new_empty((4, 4)))


def _rade_project_setup(ctx, inputs, output):
    means, quats, scales, opacities, view, full, K, width, height, *_, kernel_size = inputs
    ctx.save_for_backward(means, quats, scales, opacities, view, full, K, output[2])
    ctx.args = (width, height, kernel_size)


def _rade_project_backward(ctx, g_centers, g_conics, g_radii, g_tiles, g_depths, g_planes,
                           g_normals):
    means, quats, scales, opacities, view, full, K, radii = ctx.saved_tensors
    n = means.shape[0]
    zero = means.new_zeros
    grads = torch.ops.splat200.rade_project_backward(
        means, quats, scales, opacities, view, full, K, *ctx.args, radii,
        zero((n, 2)) if g_centers is None else g_centers,
        zero((n, 4)) if g_conics is None else g_conics,
        zero((n, 3)) if g_planes is None else g_planes,
        zero((n, 3)) if g_normals is None else g_normals)
    return (*grads, None, None, None, None, None, None, None)


rade_project.register_autograd(_rade_project_backward, setup_context=_rade_project_setup)


@torch.library.custom_op(f"{_NS}::rade_render", mutates_args=())
def rade_render(centers: Tensor, conics: Tensor, planes: Tensor, normals: Tensor,
                ranges: Tensor, point_list: Tensor, features: Tensor, background: Tensor,
                K: Tensor, width: int, height: int
                ) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """features (N, C) and background (C).  Returns the features (H, W, C),
    alpha, expected depth and median depth (H, W, 1), normals (H, W, 3),
    auxiliary (2, H, W) and contributors (2, H, W)."""
    from .rade import projection as rp
    from .rade import render as rr
    st = rp.ProjectedGaussians(centers, conics, None, None, None, planes, normals)
    out = rr.render(st, dict(ranges=ranges, point_list=point_list), features, None,
                    background, K, width, height)
    return (out.features, out.alpha, out.depth, out.median, out.normals, out.auxiliary,
            out.contributors)


@rade_render.register_fake
def _(centers, conics, planes, normals, ranges, point_list, features, background, K, width,
      height):
    C = features.shape[1]
    img = features.new_empty
    return (img((height, width, C)), img((height, width, 1)), img((height, width, 1)),
            img((height, width, 1)), img((height, width, 3)), img((2, height, width)),
            img((2, height, width), dtype=torch.int32))


@torch.library.custom_op(f"{_NS}::rade_render_backward", mutates_args=())
def rade_render_backward(centers: Tensor, conics: Tensor, planes: Tensor, normals: Tensor,
                         ranges: Tensor, point_list: Tensor, features: Tensor,
                         background: Tensor, K: Tensor, alpha: Tensor, normal_image: Tensor,
                         auxiliary: Tensor, contributors: Tensor, grad_features: Tensor,
                         grad_alpha: Tensor, grad_depth: Tensor, grad_median: Tensor,
                         grad_normals: Tensor, width: int, height: int
                         ) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Gradients of centers, conics, ray planes, normals, features and the
    |d centers| sums."""
    from .rade import projection as rp
    from .rade import render as rr
    st = rp.ProjectedGaussians(centers, conics, None, None, None, planes, normals)
    fwd = rr.RenderedPixels(None, alpha, None, None, normal_image, auxiliary, contributors)
    gc, gq, gf, _, gp, gn, gabs = rr.backward(
        st, dict(ranges=ranges, point_list=point_list), features, None, background, K, fwd,
        (grad_features, grad_alpha, grad_depth, grad_median, grad_normals), width, height,
        absgrad=True)
    return gc, gq, gp, gn, gf, gabs


@rade_render_backward.register_fake
def _(centers, conics, planes, normals, ranges, point_list, features, background, K, alpha,
      normal_image, auxiliary, contributors, grad_features, grad_alpha, grad_depth,
      grad_median, grad_normals, width, height):
    return (torch.empty_like(centers), torch.empty_like(conics), torch.empty_like(planes),
            torch.empty_like(normals), torch.empty_like(features), torch.empty_like(centers))


def _rade_render_setup(ctx, inputs, output):
    centers, conics, planes, normals, ranges, point_list, features, background, K, W, H = inputs
    ctx.save_for_backward(centers, conics, planes, normals, ranges, point_list, features,
                          background, K, output[1], output[4], output[5], output[6])
    ctx.size = (W, H)


def _rade_render_backward(ctx, g_feat, g_alpha, g_depth, g_median, g_normals, g_aux,
                          g_contrib):
    (centers, conics, planes, normals, ranges, point_list, features, background, K, alpha,
     normal_image, aux, contrib) = ctx.saved_tensors
    W, H = ctx.size
    zero = features.new_zeros

    def up(g, k):
        return zero((H, W, k)) if g is None else g.contiguous()

    gc, gq, gp, gn, gf, _ = torch.ops.splat200.rade_render_backward(
        centers, conics, planes, normals, ranges, point_list, features, background, K, alpha,
        normal_image, aux, contrib, up(g_feat, features.shape[1]), up(g_alpha, 1),
        up(g_depth, 1), up(g_median, 1), up(g_normals, 3), W, H)
    return gc, gq, gp, gn, None, None, gf, None, None, None, None


rade_render.register_autograd(_rade_render_backward, setup_context=_rade_render_setup)

OPERATORS = ("cameras_prepare", "project", "project_backward", "project_views",
             "project_views_backward", "sh_forward", "sh_backward", "bin_and_sort", "render",
             "render_backward", "rade_project", "rade_project_backward", "rade_render",
             "rade_render_backward")
