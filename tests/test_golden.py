"""The oracle against golden vectors from dsl_splat's own kernels.

tests/golden/gs3d_*.npz hold inputs and outputs of the reference's gs3d
kernels (camera prep and VJP, projection, SH forward/backward, metadata,
duplicate + stable sort + identify_ranges, blend forward and backward),
executed on the CPU through tests/golden/warp_shim.py by make_golden.py.
The oracle restates the same kernels; expected agreement:
  * integers (radii, tile counts, keys, ids, ranges, contributors) and the
    float outputs computed with the same operation sequence (projection,
    SH forward, metadata, camera rows, transmittance, colours) -- bit-exact;
  * camera centres -- Warp's 4x4 inverse is not restated bit for bit
    (relative 1e-6);
  * gradients -- relative L2 1e-5 (float32 atomics in thread order against
    the oracle's float64 sums; SH direction gradients against a finite-
    difference Warp autodiff stand-in: 1e-4).
"""

import glob
import os

import numpy as np
import pytest

from conftest import ROOT, rel_l2
from oracle import oracle as O

FIXTURES = sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "gs3d_*.npz")))


def _load(path):
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(params=FIXTURES, ids=[os.path.basename(p)[5:-4] for p in FIXTURES])
def golden(request):
    return _load(request.param)


def test_fixtures_present():
    assert len(FIXTURES) >= 2


def test_cameras(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    full, inverse, campos, err = O.cameras_prepare(g["viewmat"][None], g["K"][None], W, H, True)
    assert err[0] == 0
    np.testing.assert_array_equal(full[0], g["full"])
    np.testing.assert_allclose(campos[0], g["campos"], rtol=1e-6, atol=1e-6)
    gv = O.cameras_backward(g["K"][None], g["cam_grad_full"][None], W, H, g["inverse"][None],
                            g["cam_grad_centers"][None])
    np.testing.assert_array_equal(gv[0], g["cam_grad_views"])


def test_projection(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    p = O.project_forward(g["means"], g["quats"], g["scales"], g["opacities"], g["viewmat"],
                          g["full"], g["K"], W, H)
    np.testing.assert_array_equal(p.radii, g["radii"])
    np.testing.assert_array_equal(p.tiles, g["tiles"])
    vis = g["radii"] > 0
    np.testing.assert_array_equal(p.centers[vis], g["centers"][vis])
    np.testing.assert_array_equal(p.conics[vis], g["conics"][vis])
    np.testing.assert_array_equal(p.depths[vis], g["depths"][vis])


def test_sh_forward_and_backward(golden):
    g = golden
    deg = int(g["sh_degree"])
    colors, active = O.sh_forward(g["sh"], g["dirs"], deg, g["radii"])
    np.testing.assert_array_equal(colors, g["colors"])
    np.testing.assert_array_equal(active.astype(bool), g["active"])
    gsh, gdir = O.sh_backward(g["sh"], g["dirs"], deg, g["radii"], active, g["sh_upstream"],
                              need_dirs=True)
    np.testing.assert_array_equal(gsh, g["grad_sh"])
    if deg > 0:
        assert rel_l2(gdir, g["grad_dirs"]) <= 1e-4


def test_binning(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    offsets, m = O.scan_counts(g["tiles"])
    np.testing.assert_array_equal(offsets, g["offsets"])
    keys, ids, ranges = O.bin_and_sort(g["centers"], g["radii"], g["depths"], offsets, W, H)
    np.testing.assert_array_equal(keys, g["keys"])
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_array_equal(ranges, g["ranges"])


def test_render_forward(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    image, final_t, contrib = O.render_forward(W, H, g["ranges"], g["ids"], g["centers"],
                                               g["conics"], g["features"], g["background"])
    np.testing.assert_array_equal(contrib, g["contributors"])
    np.testing.assert_array_equal(final_t, g["final_t"])
    np.testing.assert_array_equal(image, g["image"])


def test_render_backward(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    gc, gq, gf, ga = O.render_backward(W, H, g["ranges"], g["ids"], g["centers"], g["conics"],
                                       g["features"], g["background"], g["final_t"],
                                       g["contributors"], g["upstream"], absgrad=True,
                                       constant_tail=1)
    assert rel_l2(gc, g["grad_centers"]) <= 1e-5
    assert rel_l2(gq, g["grad_conics"]) <= 1e-5
    assert rel_l2(gf, g["grad_features"]) <= 1e-5
    assert rel_l2(ga, g["grad_abs"]) <= 1e-5


def test_metadata(golden):
    g = golden
    vis = g["radii"] > 0
    np.testing.assert_array_equal(g["meta_means2d"][vis], g["centers"][vis])
    assert not g["meta_means2d"][~vis].any()
    np.testing.assert_array_equal(g["meta_opacities"][vis], g["conics"][vis, 3])


TILE_MODE_FIXTURES = sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "tilemodes_*.npz")))


@pytest.mark.parametrize("path", TILE_MODE_FIXTURES,
                         ids=[os.path.basename(p)[10:-4] for p in TILE_MODE_FIXTURES])
@pytest.mark.parametrize("mode", ["snugbox", "accutile"])
def test_tile_modes(path, mode):
    """tile_mode snugbox/accutile (splatting/intersections.py:45-218 through
    gs3d/projection.py:150-162 and splatting/binning.py:40-117): tile counts,
    sorted keys, ids and ranges bit-exact."""
    g = _load(path)
    W, H = int(g["width"]), int(g["height"])
    p = O.project_forward(g["means"], g["quats"], g["scales"], g["opacities"], g["viewmat"],
                          g["full"], g["K"], W, H, tile_mode=mode)
    np.testing.assert_array_equal(p.radii, g[f"{mode}_radii"])
    np.testing.assert_array_equal(p.tiles, g[f"{mode}_tiles"])
    vis = p.radii > 0
    np.testing.assert_array_equal(p.conics[vis], g[f"{mode}_conics"][vis])
    off, _ = O.scan_counts(p.tiles)
    keys, ids, ranges = O.bin_and_sort(p.centers, p.radii, p.depths, off, W, H,
                                       conics=p.conics, tile_mode=mode)
    np.testing.assert_array_equal(keys, g[f"{mode}_keys"])
    np.testing.assert_array_equal(ids, g[f"{mode}_ids"])
    np.testing.assert_array_equal(ranges, g[f"{mode}_ranges"])


def test_tile_mode_fixtures_present():
    assert len(TILE_MODE_FIXTURES) == 3


WIDE_FIXTURES = sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "wide_*.npz")))


@pytest.mark.parametrize("path", WIDE_FIXTURES, ids=[os.path.basename(p)[5:-4]
                                                     for p in WIDE_FIXTURES])
def test_oracle_wide_blend(path):
    """Eight blended channels over a random background, forward and backward:
    the oracle against the reference's own kernels."""
    with np.load(path) as z:
        g = {k: z[k] for k in z.files}
    W, H = int(g["width"]), int(g["height"])
    image, final_t, contrib = O.render_forward(W, H, g["ranges"], g["ids"], g["centers"],
                                               g["conics"], g["features"], g["background"])
    np.testing.assert_array_equal(contrib, g["contributors"])
    np.testing.assert_array_equal(final_t, g["final_t"])
    assert np.abs(image - g["image"]).max() <= 1e-5
    gc, gq, gf, ga = O.render_backward(W, H, g["ranges"], g["ids"], g["centers"], g["conics"],
                                       g["features"], g["background"], g["final_t"],
                                       g["contributors"], g["upstream"], absgrad=True,
                                       constant_tail=1)
    assert rel_l2(gc, g["grad_centers"]) <= 1e-5
    assert rel_l2(gq, g["grad_conics"]) <= 1e-5
    assert rel_l2(gf, g["grad_features"]) <= 1e-5
    assert rel_l2(ga, g["grad_abs"]) <= 1e-5


# ---- projection VJP against float64 autograd with the reference's adjoints --
#
# The reference differentiates projection_loss (gs3d/projection.py:198-210)
# with Warp autodiff, which the shim cannot run; the oracle's VJP is
# hand-derived.  This restates projection_loss in float64 Torch, with the
# reference's three custom adjoints as autograd Functions, and checks the
# oracle's gradients against autograd's.

import torch  # noqa: E402


class _Rotation(torch.autograd.Function):
    """glm_rotation (primitives/math.py:33-45) with adj_reference_rotation
    (splatting/math.py:13-28)."""

    @staticmethod
    def forward(ctx, q):
        ctx.save_for_backward(q)
        r, x, y, z = q.unbind(-1)
        rows = [[1 - 2 * (y * y + z * z), 2 * (x * y + r * z), 2 * (x * z - r * y)],
                [2 * (x * y - r * z), 1 - 2 * (x * x + z * z), 2 * (y * z + r * x)],
                [2 * (x * z + r * y), 2 * (y * z - r * x), 1 - 2 * (x * x + y * y)]]
        return torch.stack([torch.stack(row, -1) for row in rows], -2)

    @staticmethod
    def backward(ctx, g):
        (q,) = ctx.saved_tensors
        r, x, y, z = q.unbind(-1)
        G = lambda i, j: g[..., i, j]  # noqa: E731
        return torch.stack([
            2 * (z * (G(0, 1) - G(1, 0)) + y * (G(2, 0) - G(0, 2)) + x * (G(1, 2) - G(2, 1))),
            2 * (y * (G(0, 1) + G(1, 0)) + z * (G(0, 2) + G(2, 0)) + r * (G(1, 2) - G(2, 1)))
            - 4 * x * (G(1, 1) + G(2, 2)),
            2 * (x * (G(0, 1) + G(1, 0)) + r * (G(2, 0) - G(0, 2)) + z * (G(1, 2) + G(2, 1)))
            - 4 * y * (G(0, 0) + G(2, 2)),
            2 * (r * (G(0, 1) - G(1, 0)) + x * (G(0, 2) + G(2, 0)) + y * (G(1, 2) + G(2, 1)))
            - 4 * z * (G(0, 0) + G(1, 1))], -1)


class _Clamp(torch.autograd.Function):
    """clamp_point with adj_clamp_point (splatting/geometry.py:33-51)."""

    @staticmethod
    def forward(ctx, t, limx, limy):
        x, y = t[:, 0] / t[:, 2], t[:, 1] / t[:, 2]
        ctx.save_for_backward((x >= -limx) & (x <= limx), (y >= -limy) & (y <= limy))
        return torch.stack([x.clamp(-limx, limx) * t[:, 2], y.clamp(-limy, limy) * t[:, 2],
                            t[:, 2]], -1)

    @staticmethod
    def backward(ctx, g):
        in_x, in_y = ctx.saved_tensors
        return torch.stack([g[:, 0] * in_x, g[:, 1] * in_y, g[:, 2]], -1), None, None


class _Inverse(torch.autograd.Function):
    """invert_covariance with adj_invert_covariance (geometry.py:54-71)."""

    @staticmethod
    def forward(ctx, cov):
        ctx.save_for_backward(cov)
        a, b, c = cov.unbind(-1)
        inv = 1.0 / (a * c - b * b)
        return torch.stack([c * inv, -b * inv, a * inv], -1)

    @staticmethod
    def backward(ctx, g):
        (cov,) = ctx.saved_tensors
        a, b, c = cov.unbind(-1)
        det = a * c - b * b
        f = 1.0 / (det * det + 1e-7)
        x, y, z = g.unbind(-1)
        return f[:, None] * torch.stack([
            -c * c * x + b * c * y + (det - a * c) * z,
            2 * b * c * x - (det + 2 * b * b) * y + 2 * a * b * z,
            -a * a * z + a * b * y + (det - a * c) * x], -1)


def _projection_loss(means, quats, scales, opac, view, proj, K, W, H, seed_c, seed_q):
    """gs3d/projection.py:37-86 screen_covariance + 198-210 projection_loss."""
    fx, fy = K[0, 0], K[1, 1]
    pos = means @ view[:3, :3].T + view[:3, 3]
    t = _Clamp.apply(pos, 1.3 * W / (2 * fx), 1.3 * H / (2 * fy))
    R = _Rotation.apply(quats)
    M = scales[:, :, None] * R                       # scaling @ rotation
    cov = M.transpose(1, 2) @ M
    z = t[:, 2]
    zero = torch.zeros_like(z)
    J = torch.stack([torch.stack([fx / z, zero, zero], -1),
                     torch.stack([zero, fy / z, zero], -1),
                     torch.stack([-(fx * t[:, 0]) / (z * z), -(fy * t[:, 1]) / (z * z), zero],
                                 -1)], -2)
    camera = view[:3, :3].T                          # rows (v00, v10, v20), ...
    T = camera @ J
    P = (T.transpose(1, 2) @ cov.transpose(1, 2)) @ T
    conic3 = _Inverse.apply(torch.stack([P[:, 0, 0] + 0.3, P[:, 1, 0], P[:, 1, 1] + 0.3], -1))
    clip = means @ proj[:, :3].T + proj[:, 3]
    inv_w = 1.0 / (clip[:, 3] + 1e-7)
    center = torch.stack([((clip[:, 0] * inv_w + 1) * W - 1) * 0.5,
                          ((clip[:, 1] * inv_w + 1) * H - 1) * 0.5], -1)
    conic = torch.cat([conic3, opac[:, None]], -1)
    return (center * seed_c).sum() + (conic * seed_q).sum()


@pytest.mark.parametrize("path", FIXTURES, ids=[os.path.basename(p)[5:-4] for p in FIXTURES])
def test_projection_vjp_against_float64_autograd(path):
    g = _load(path)
    W, H = int(g["width"]), int(g["height"])
    vis = g["radii"] > 0
    n = len(g["means"])
    rng = np.random.default_rng(7)
    seed_c = rng.standard_normal((n, 2)).astype(np.float32)
    seed_q = (rng.standard_normal((n, 4)) * 1e-2).astype(np.float32)
    gm, gq, gs, go, gv, gp = O.project_backward(
        g["means"], g["quats"], g["scales"], g["opacities"], g["viewmat"], g["full"], g["K"],
        W, H, g["radii"], seed_c, seed_q)

    def t(a, grad=False):
        return torch.tensor(np.asarray(a, np.float64), requires_grad=grad)

    leaves = [t(g[k][vis], True) for k in ("means", "quats", "scales", "opacities")]
    view, proj = t(g["viewmat"], True), t(g["full"], True)
    loss = _projection_loss(*leaves, view, proj, t(g["K"]), W, H, t(seed_c[vis]),
                            t(seed_q[vis]))
    loss.backward()
    for got, leaf, name in zip((gm, gq, gs, go), leaves, ("means", "quats", "scales", "op")):
        assert not np.asarray(got)[~vis].any(), name  # culled rows stay zero
        assert rel_l2(np.asarray(got)[vis], leaf.grad.numpy()) <= 1e-5, name
    assert rel_l2(gv, view.grad.numpy()) <= 1e-5
    assert rel_l2(gp, proj.grad.numpy()) <= 1e-5
