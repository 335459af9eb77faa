"""The sm_100a kernels (through the C ABI) against golden vectors from
dsl_splat's own kernels (tests/golden, see make_golden.py).

Same tolerances as the oracle parity tests: integers and the projection /
SH / camera floats bit-exact, transmittance and contributors bit-exact,
images max-abs 1e-5, gradients relative L2 1e-3.
"""

import glob
import os

import numpy as np
import pytest
import torch

from conftest import ROOT, rel_l2
from dsl_splat_b200 import stages

pytestmark = pytest.mark.gpu

FIXTURES = sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "gs3d_*.npz")))


@pytest.fixture(params=FIXTURES, ids=[os.path.basename(p)[5:-4] for p in FIXTURES])
def golden(request):
    with np.load(request.param) as z:
        return {k: z[k] for k in z.files}


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")
    return t if dtype is None else t.to(dtype)


def test_gpu_matches_reference_kernels(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    deg = int(g["sh_degree"])
    full, inv, campos = stages.cameras_prepare(_t(g["viewmat"])[None], _t(g["K"])[None], W, H, True)
    np.testing.assert_array_equal(full[0].cpu().numpy(), g["full"])
    np.testing.assert_allclose(campos[0].cpu().numpy(), g["campos"], rtol=1e-6, atol=1e-6)
    # SH directions use the reference's camera centre so colours can match bit for bit
    out = stages.project_fused(_t(g["means"]), _t(g["quats"]), _t(g["scales"]),
                               _t(g["opacities"]), _t(g["viewmat"]), _t(g["full"]), _t(g["K"]),
                               W, H, 0.2, float("inf"), 0.0, sh=_t(g["sh"]), sh_degree=deg,
                               campos=_t(g["campos"]))
    st = out.state
    radii = st.radii.cpu().numpy()
    np.testing.assert_array_equal(radii, g["radii"])
    np.testing.assert_array_equal(st.tile_counts.cpu().numpy(), g["tiles"])
    vis = radii > 0
    np.testing.assert_array_equal(st.centers.cpu().numpy()[vis], g["centers"][vis])
    np.testing.assert_array_equal(st.conics.cpu().numpy()[vis], g["conics"][vis])
    np.testing.assert_array_equal(st.depths.cpu().numpy()[vis], g["depths"][vis])
    np.testing.assert_array_equal(out.colors.cpu().numpy(), g["colors"])
    np.testing.assert_array_equal(out.active.cpu().numpy().astype(bool), g["active"])
    np.testing.assert_array_equal(out.means2d.cpu().numpy(), g["meta_means2d"])

    bins = stages.bin_and_sort(st, W, H)
    np.testing.assert_array_equal(bins["ranges"].cpu().numpy(), g["ranges"])
    np.testing.assert_array_equal(bins["point_list"].cpu().numpy(), g["ids"])

    bg = _t(g["background"])
    px = stages.render(st, bins, out.colors, None, True, bg, W, H)
    np.testing.assert_array_equal(px.contributors.cpu().numpy(), g["contributors"])
    np.testing.assert_array_equal(px.transmittance.cpu().numpy(), g["final_t"])
    img = np.moveaxis(px.features.cpu().numpy(), -1, 0)
    assert np.abs(img - g["image"]).max() <= 1e-5

    up = _t(np.moveaxis(g["upstream"], 0, -1))
    gc, gq, ga, _, gabs = stages.render_backward(st, bins, out.colors, None, True, bg,
                                                 px.transmittance, px.contributors, up, W, H,
                                                 absgrad=True, constant_tail=1)
    assert rel_l2(gc.cpu(), g["grad_centers"]) <= 1e-3
    assert rel_l2(gq.cpu(), g["grad_conics"]) <= 1e-3
    assert rel_l2(ga.cpu(), g["grad_features"][:, :3]) <= 1e-3
    assert rel_l2(gabs.cpu(), g["grad_abs"]) <= 1e-3

    gsh, gdir = stages.sh_backward(_t(g["sh"]), _t(g["dirs"]), deg, st.radii, out.active,
                                   _t(g["sh_upstream"]), True)
    np.testing.assert_array_equal(gsh.cpu().numpy(), g["grad_sh"])
    if deg > 0:
        assert rel_l2(gdir.cpu(), g["grad_dirs"]) <= 1e-3

    gv = stages.cameras_backward(_t(g["K"])[None], _t(g["cam_grad_full"])[None], W, H,
                                 _t(g["inverse"])[None], _t(g["cam_grad_centers"])[None],
                                 (1, 4, 4))
    np.testing.assert_array_equal(gv[0].cpu().numpy(), g["cam_grad_views"])


TILE_MODE_FIXTURES = sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "tilemodes_*.npz")))


@pytest.mark.parametrize("path", TILE_MODE_FIXTURES,
                         ids=[os.path.basename(p)[10:-4] for p in TILE_MODE_FIXTURES])
@pytest.mark.parametrize("mode", ["snugbox", "accutile"])
def test_gpu_tile_modes_match_reference_kernels(path, mode):
    """tile_mode snugbox/accutile through the C ABI: projection tile counts,
    point_list and ranges bit-exact with the reference's intersection
    kernels (splatting/intersections.py:45-218)."""
    with np.load(path) as z:
        g = {k: z[k] for k in z.files}
    W, H = int(g["width"]), int(g["height"])
    st = stages.project(_t(g["means"]), _t(g["quats"]), _t(g["scales"]), _t(g["opacities"]),
                        _t(g["viewmat"]), _t(g["full"]), _t(g["K"]), W, H, 0.2, float("inf"),
                        0.0, tile_mode=mode)
    radii = st.radii.cpu().numpy()
    np.testing.assert_array_equal(radii, g[f"{mode}_radii"])
    np.testing.assert_array_equal(st.tile_counts.cpu().numpy(), g[f"{mode}_tiles"])
    vis = radii > 0
    np.testing.assert_array_equal(st.conics.cpu().numpy()[vis], g[f"{mode}_conics"][vis])
    bins = stages.bin_and_sort(st, W, H, tile_mode=mode)
    np.testing.assert_array_equal(bins["ranges"].cpu().numpy(), g[f"{mode}_ranges"])
    np.testing.assert_array_equal(bins["point_list"].cpu().numpy(), g[f"{mode}_ids"])


WIDE_FIXTURES = sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "wide_*.npz")))


@pytest.mark.parametrize("path", WIDE_FIXTURES, ids=[os.path.basename(p)[5:-4]
                                                     for p in WIDE_FIXTURES])
def test_gpu_wide_blend_and_statistics(path):
    """Eight channels (colours, four extras, the constant one) over a random
    background with a masked-count and a weighted-sum statistics request,
    forward and backward, against the reference's own kernels."""
    from dsl_splat_b200.statistics import PreparedStatistics
    with np.load(path) as z:
        g = {k: z[k] for k in z.files}
    W, H = int(g["width"]), int(g["height"])
    n = len(g["centers"])
    st = stages.ProjectedFootprint(_t(g["centers"]), _t(g["conics"]))
    bins = dict(ranges=_t(g["ranges"]), point_list=_t(g["ids"]))
    feats = g["features"]
    a, b, bg = _t(feats[:, :3]), _t(feats[:, 3:7]), _t(g["background"])
    stats = PreparedStatistics(
        key=(0, 1), pixel_values=_t(np.stack([g["mask"].ravel(), g["weights"].ravel()])),
        counts=torch.zeros((1, n), dtype=torch.int32, device="cuda:0"),
        sums=torch.zeros((1, n), device="cuda:0"))
    px = stages.render(st, bins, a, b, True, bg, W, H, planar=True, statistics=stats)
    np.testing.assert_array_equal(px.contributors.cpu().numpy(), g["contributors"])
    np.testing.assert_array_equal(px.transmittance.cpu().numpy(), g["final_t"])
    assert np.abs(px.features.cpu().numpy() - g["image"]).max() <= 1e-5
    np.testing.assert_array_equal(stats.counts[0].cpu().numpy(), g["stat_counts"])
    assert rel_l2(stats.sums[0].cpu().numpy(), g["stat_sums"]) <= 1e-5
    gc, gq, ga, gb, gabs = stages.render_backward(
        st, bins, a, b, True, bg, px.transmittance, px.contributors, _t(g["upstream"]), W, H,
        planar=True, absgrad=True, constant_tail=1)
    assert rel_l2(gc.cpu(), g["grad_centers"]) <= 1e-3
    assert rel_l2(gq.cpu(), g["grad_conics"]) <= 1e-3
    assert rel_l2(ga.cpu(), g["grad_features"][:, :3]) <= 1e-3
    assert rel_l2(gb.cpu(), g["grad_features"][:, 3:7]) <= 1e-3
    assert rel_l2(gabs.cpu(), g["grad_abs"]) <= 1e-3
