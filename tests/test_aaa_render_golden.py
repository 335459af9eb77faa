"""The AAA hierarchical blend oracle against the reference's own kernels.

tests/golden/aaa_render_*.npz hold aaa/render_hierarchical_warp.py's render
(HIER 64/8/4 queues, 3D ray evaluation, 4x4 culling) and
aaa/backward_render.py's replay, executed on the CPU through the Warp
stand-in (tests/golden/make_golden.py --aaa-render-only) on the bins of the
load-balanced preprocessing path.  The oracle (oracle/aaa_render_oracle.cpp)
must reproduce the image, final transmittance and evaluated-sample counts
bit for bit (same float32 operation order, same exp), and the replay's
gradients within 1e-4 relative L2 (the reference sums float32 atomics in
thread order, the oracle float64).
"""

import glob
import os

import numpy as np
import pytest

from conftest import ROOT, rel_l2
from oracle import oracle as O

FIXTURES = sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "aaa_render_*.npz")))


@pytest.fixture(params=FIXTURES, ids=[os.path.basename(p)[11:-4] for p in FIXTURES])
def golden(request):
    with np.load(request.param) as z:
        return {k: z[k] for k in z.files}


def test_hier_blend_bit_exact(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    image, final_t, contrib = O.aaa_render(W, H, g["ranges"], g["ids"], g["transforms"],
                                           g["opacity"], g["features"], g["background"],
                                           cull=bool(g["cull"]))
    np.testing.assert_array_equal(contrib, g["contributors"])
    np.testing.assert_array_equal(final_t, g["final_t"])
    np.testing.assert_array_equal(image, g["image"])
    assert contrib.max() > 0


def test_hier_statistics(golden):
    """render_statistics (render_hierarchical_warp.py:608-653, the observer of
    statistics.py:47-73): a masked count bit for bit, a weighted sum within
    1e-6 relative L2 (the reference adds float32 products atomically)."""
    g = golden
    if "stat_counts" not in g:
        pytest.skip("this golden has no statistics requests")
    W, H = int(g["width"]), int(g["height"])
    maps = np.stack([g["stat_mask"], g["stat_weights"]])
    image, final_t, contrib, counts, sums = O.aaa_render(
        W, H, g["ranges"], g["ids"], g["transforms"], g["opacity"], g["features"],
        g["background"], cull=bool(g["cull"]), stat_maps=maps, stat_kinds=(0, 1))
    np.testing.assert_array_equal(image, g["image"])
    np.testing.assert_array_equal(counts[0], g["stat_counts"])
    assert g["stat_counts"].any() and g["stat_sums"].any()
    assert rel_l2(sums[0], g["stat_sums"]) <= 1e-6


def test_hier_replay_gradients(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    got = O.aaa_render_backward(W, H, g["ranges"], g["ids"], g["transforms"], g["opacity"],
                                g["features"], g["background"], g["image"], g["final_t"],
                                g["upstream"], cull=bool(g["cull"]), screen=True, absgrad=True)
    for key, ref in (("transforms", "grad_transforms"), ("opacity", "grad_opacity"),
                     ("colors", "grad_features"), ("screen", "grad_screen"),
                     ("screen_abs", "grad_screen_abs")):
        assert np.abs(g[ref]).sum() > 0, ref
        assert rel_l2(got[key], g[ref]) <= 1e-4, key
    # the depth column of every transform gradient row stays zero
    # (render_adjoint.py:313-314: CUDA's float4 blocks skip screen depth)
    assert not got["transforms"].reshape(-1, 4, 4)[:, :, 2].any()
