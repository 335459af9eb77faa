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
