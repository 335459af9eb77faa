"""The RaDe-GS oracle against golden vectors from dsl_splat's own rade
kernels (tests/golden/rade_*.npz, made by make_golden.py --rade-only:
rade/projection.py:194-260 project, splatting/binning.py duplicate with the
radial depths, rade/render.py:99-322 render and :325-547 backward, run on
the CPU Warp stand-in).

Expected agreement: projection outputs, bins, images, auxiliary planes and
contributors bit-exact (same float32 operation sequence); render gradients
relative L2 1e-5 (the reference's warp-reduced float32 atomics against the
oracle's float64 sums).  The projection VJP oracle (float64 autograd with
the reference's custom adjoints, oracle/rade_vjp.py) is checked for its
structure here and against the CUDA backward in the GPU tests.
"""

import glob
import os

import numpy as np
import pytest
import torch

from conftest import ROOT, rel_l2
from oracle import oracle as O
from oracle import rade_vjp

FIXTURES = sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "rade_*.npz")))


@pytest.fixture(params=FIXTURES, ids=[os.path.basename(p)[5:-4] for p in FIXTURES])
def golden(request):
    with np.load(request.param) as z:
        return {k: z[k] for k in z.files}


def features_of(g):
    return np.concatenate([g["colors"], g["extras"]], axis=1).astype(np.float32)


def test_fixtures_present():
    assert len(FIXTURES) >= 3


def test_rade_projection(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    p = O.rade_project(g["means"], g["quats"], g["scales"], g["opacities"], g["viewmat"],
                       g["full"], g["K"], W, H, kernel_size=float(g["kernel_size"]))
    np.testing.assert_array_equal(p["radii"], g["radii"])
    np.testing.assert_array_equal(p["tiles"], g["tiles"])
    vis = g["radii"] > 0
    for k in ("centers", "conics", "depths", "planes", "normals"):
        np.testing.assert_array_equal(p[k][vis], g[k][vis], err_msg=k)


def test_rade_bins(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    offsets = np.cumsum(g["tiles"]).astype(np.int32)
    keys, ids, ranges = O.bin_and_sort(g["centers"], g["radii"], g["depths"], offsets, W, H)
    np.testing.assert_array_equal(keys, g["keys"])
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_array_equal(ranges, g["ranges"])


def test_rade_render(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    image, aux, contrib = O.rade_render(W, H, g["ranges"], g["ids"], g["centers"], g["conics"],
                                        features_of(g), g["background"], g["planes"],
                                        g["normals"], g["K"])
    np.testing.assert_array_equal(image, g["image"])
    np.testing.assert_array_equal(aux, g["auxiliary"])
    np.testing.assert_array_equal(contrib, g["contributors"])


def test_rade_render_backward(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    out = O.rade_render_backward(
        W, H, g["ranges"], g["ids"], g["centers"], g["conics"], features_of(g), g["background"],
        g["planes"], g["normals"], g["K"], g["image"], g["auxiliary"], g["contributors"],
        g["up_features"], g["up_alpha"], g["up_depth"], g["up_median"], g["up_normals"])
    for ours, ref in (("centers", "grad_centers"), ("conics", "grad_conics"),
                      ("features", "grad_features"), ("abs", "grad_abs"),
                      ("planes", "grad_planes"), ("normals", "grad_normals")):
        assert rel_l2(out[ours], g[ref]) <= 1e-5, ours


def test_rade_median_and_depth_semantics(golden):
    """rade/render.py:197-227: the median contributor is never after the
    last; expected depth is zero where nothing blended; alpha = 1 - T."""
    g = golden
    C = g["image"].shape[0] - 6
    last, median = g["contributors"]
    assert (median <= last).all()
    assert ((median == -1) | (median >= 1)).all()
    nothing = last == 0
    assert (g["image"][C + 1][nothing] == 0).all()
    assert (g["image"][C][nothing] == 0).all()


def test_rade_vjp_oracle_structure(golden):
    """Culled rows get zero gradients; seeds on planes/normals of rows in
    the degenerate-direction branch contribute nothing; a zero seed gives
    zero gradients."""
    g = golden
    W, H = int(g["width"]), int(g["height"])
    n = len(g["means"])
    rng = np.random.default_rng(11)
    seeds = [rng.standard_normal((n, k)).astype(np.float32) for k in (2, 4, 3, 3)]
    seeds[1] *= 1e-2
    grads = rade_vjp.project_backward(g["means"], g["quats"], g["scales"], g["opacities"],
                                      g["viewmat"], g["full"], g["K"], W, H, g["radii"], *seeds,
                                      kernel_size=float(g["kernel_size"]), planes=g["planes"])
    vis = g["radii"] > 0
    for grad in grads[:4]:
        assert np.isfinite(grad).all()
        assert not grad[~vis].any()
    zero = [np.zeros_like(s) for s in seeds]
    grads0 = rade_vjp.project_backward(g["means"], g["quats"], g["scales"], g["opacities"],
                                       g["viewmat"], g["full"], g["K"], W, H, g["radii"], *zero,
                                       kernel_size=float(g["kernel_size"]), planes=g["planes"])
    assert all(not np.asarray(x).any() for x in grads0)


def test_rade_vjp_oracle_matches_finite_differences_without_custom_adjoints():
    """Through the centre and ray-plane seeds alone (no custom adjoint on
    their path except the rotation, whose adjoint is the exact derivative of
    glm_rotation on unit quaternions' tangent space), the float64 autograd
    oracle agrees with central differences of the same loss."""
    g = dict(np.load(FIXTURES[0]))
    W, H = int(g["width"]), int(g["height"])
    vis = np.flatnonzero(g["radii"] > 0)[:5]
    rng = np.random.default_rng(5)
    k = len(vis)
    seeds = (torch.tensor(rng.standard_normal((k, 2))), torch.zeros((k, 4), dtype=torch.float64),
             torch.tensor(rng.standard_normal((k, 3))), torch.zeros((k, 3), dtype=torch.float64))

    def loss(means):
        return rade_vjp.projection_loss(
            means, torch.tensor(g["quats"][vis], dtype=torch.float64),
            torch.tensor(g["scales"][vis], dtype=torch.float64),
            torch.tensor(g["opacities"][vis], dtype=torch.float64),
            torch.tensor(g["viewmat"], dtype=torch.float64),
            torch.tensor(g["full"], dtype=torch.float64),
            torch.tensor(g["K"], dtype=torch.float64), W, H, 0.0, seeds, g["scales"][vis])

    means = torch.tensor(g["means"][vis], dtype=torch.float64, requires_grad=True)
    loss(means).backward()
    fd = np.zeros((k, 3))
    h = 1e-6
    for i in range(k):
        for j in range(3):
            up, dn = means.detach().clone(), means.detach().clone()
            up[i, j] += h
            dn[i, j] -= h
            fd[i, j] = (loss(up).item() - loss(dn).item()) / (2 * h)
    assert rel_l2(means.grad.numpy(), fd) <= 1e-5


def test_rade_api_validation_cpu():
    """Argument checks run before any device work (rade/api.py:82-99,
    rade/gsplat.py:17-79, rade/filtering.py:7-26)."""
    from dsl_splat_b200 import rade
    from dsl_splat_b200.rade.gsplat import rasterization

    x = torch.zeros(1, 3)
    with pytest.raises(ValueError, match="kernel_size"):
        rade.rasterize(x, x, x, x, x, x, 4, 4, features=x, kernel_size=-1.0)
    with pytest.raises(ValueError, match="kernel_size"):
        rade.rasterize(x, x, x, x, x, x, 4, 4, features=x, kernel_size=float("nan"))
    with pytest.raises(ValueError, match="eps2d"):
        rasterization(x, x, x, x, x, x, x, 4, 4, eps2d=-0.1)
    with pytest.raises(ValueError, match="render_mode"):
        rasterization(x, x, x, x, x, x, x, 4, 4, render_mode="RGB+N")
    with pytest.raises(NotImplementedError, match="with_eval3d"):
        rasterization(x, x, x, x, x, x, x, 4, 4, with_eval3d=True)
    with pytest.raises(ValueError, match="filter_3d"):
        rade.apply_3d_filter(torch.ones(5, 3), torch.ones(5), torch.ones(5))
    s, o = rade.apply_3d_filter(torch.full((2, 3), 0.3), torch.full((2,), 0.5),
                                torch.full((2, 1), 0.4))
    torch.testing.assert_close(s, torch.full((2, 3), 0.5))
    torch.testing.assert_close(o, torch.full((2,), 0.5 * (0.09 / 0.25) ** 1.5))
