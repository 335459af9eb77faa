"""The AAA-Gaussians preprocessing oracle (oracle/aaa_oracle.cpp) against
golden vectors made by executing dsl_splat's own aaa/preprocess3d.py:17-245
and, on the load-balanced cases, aaa/cooperative_culling.py:152-192 and
(aaa_coop) the key emission aaa/binning_native.py:7-135, and on every case
the preprocessing adjoint aaa/backward_preprocess.py:130-268 and the camera
adjoint aaa/backward_camera.py:61-224 with seeded upstream gradients
(tests/golden/make_golden.py --aaa-only).

Five flag sets cover every branch of preprocess_3d: the load-balanced
defaults (aaa/config.py:41-54) with and without SH colours and a stored 3D
filter, the complete path with serial tile culling, the screen-space
quadric bounds with near clipping and no EWA compensation, and no tile
culling.  Integers (radii, tile counts, valid flags, the queue of long
rectangles) are bit-exact; so is every float, because the restatement keeps
the kernel's rounding order and both sides evaluate atan2, tan and log with
the oracle's own functions (the golden generator substitutes them for the
snippets' libm calls, as it does wp.exp).
"""

import glob
import os

import numpy as np
import pytest

from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = sorted(p for p in glob.glob(os.path.join(HERE, "golden", "aaa_*.npz"))
               if not os.path.basename(p).startswith("aaa_render_"))


def _run(d, **overrides):
    flags = dict(zip(O.AAA_FLAGS, d["flags"].tolist()))
    args = dict(sh=d["sh"] if bool(d["use_sh"]) else None, sh_degree=int(d["sh_degree"]),
                filters=d["filters"] if bool(d["has_filter"]) else None, flags=flags)
    args.update(overrides)
    return O.aaa_preprocess(d["means"], d["quats"], d["scales"], d["opacities"], d["view"],
                            d["proj"], d["campos"], int(d["width"]), int(d["height"]),
                            d["tanfov"], d["principal"], **args)


def test_cases_present():
    names = {os.path.basename(c)[4:-4] for c in CASES}
    assert names == {"coop", "coop_sh3_filter", "complete", "screen_bounds", "noculling"}


@pytest.mark.parametrize("path", CASES, ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_matches_reference_kernel(path):
    d = np.load(path)
    out = _run(d)
    for key in ("radii", "tiles", "valid", "queued"):
        np.testing.assert_array_equal(out[key], d[key], err_msg=key)
    visible = d["radii"] > 0
    assert visible.any()
    for key in ("centers", "rects", "depths", "transforms", "opacity"):
        np.testing.assert_array_equal(out[key][visible], d[key][visible], err_msg=key)
    if bool(d["use_sh"]):
        np.testing.assert_array_equal(out["rgb"][visible], d["rgb"][visible])
        np.testing.assert_array_equal(out["clamped"][visible], d["clamped"][visible])
    if "final_radii" in d:
        final = O.aaa_cull_remainder(out, int(d["width"]), int(d["height"]))
        for key in ("radii", "tiles", "valid"):
            np.testing.assert_array_equal(final[key], d["final_" + key], err_msg="final " + key)
    if "dup_keys" in d:
        offsets, keys, values = O.aaa_duplicate(out, final["radii"], final["tiles"],
                                                int(d["width"]), int(d["height"]))
        np.testing.assert_array_equal(offsets, d["dup_offsets"])
        np.testing.assert_array_equal(keys, d["dup_keys"])
        np.testing.assert_array_equal(values, d["dup_values"])


def test_goldens_cover_the_branches():
    load = {os.path.basename(c)[4:-4]: np.load(c) for c in CASES}
    coop, complete = load["coop"], load["complete"]
    # long rectangles are queued on the load-balanced path only
    assert len(coop["queued"]) > 0 and len(complete["queued"]) == 0
    assert np.all(coop["radii"][coop["queued"]] > 0)
    # after the remainder cull the load-balanced counts are the complete
    # path's serial counts, and only queued rows changed
    np.testing.assert_array_equal(coop["final_tiles"], complete["tiles"])
    rest = np.setdiff1d(np.arange(len(coop["radii"])), coop["queued"])
    np.testing.assert_array_equal(coop["final_tiles"][rest], coop["tiles"][rest])
    assert np.all(coop["final_tiles"][coop["queued"]] > coop["tiles"][coop["queued"]])
    # culled groups of the scene: behind the camera, off screen, below 1/255
    for d in load.values():
        assert not d["radii"][:32].any() and not d["radii"][64:72].any()
    # valid is only set on the complete or load-balanced paths
    assert not load["noculling"]["valid"].any() and coop["valid"].sum() == (coop["radii"] > 0).sum()
    # PTD_MAX depths are camera distances on the valid rows
    v = coop["valid"]
    dist = np.linalg.norm(coop["means"][v] - coop["campos"], axis=1)
    np.testing.assert_allclose(coop["depths"][v], dist, rtol=1e-6)
    sh = load["coop_sh3_filter"]
    assert sh["clamped"][sh["valid"]].any() and not sh["clamped"][sh["valid"]].all()


def test_oracle_is_sensitive_to_its_inputs():
    """A planted change in the oracle's inputs moves its outputs (the
    comparison above is not vacuous)."""
    d = np.load(os.path.join(HERE, "golden", "aaa_coop.npz"))
    moved = dict(d)
    moved["opacities"] = d["opacities"] * np.float32(0.999)
    out = _run(moved)
    assert not np.array_equal(out["opacity"], d["opacity"])
    out = _run(d, flags=dict(zip(O.AAA_FLAGS, d["flags"].tolist()), ewa=False))
    assert not np.array_equal(out["opacity"], d["opacity"])


def test_remainder_cull_rejects_a_rectangle_without_tiles():
    """cull_remainder_3d's rejection branch (aaa/cooperative_culling.py:188-192),
    which the golden scene does not reach: a queued Gaussian whose first 32
    tiles counted none and whose threshold no tile meets loses its radius."""
    d = np.load(os.path.join(HERE, "golden", "aaa_coop.npz"))
    pre = _run(d)
    i, other = int(pre["queued"][0]), int(pre["queued"][1])
    pre["tiles"][i] = 0
    pre["opacity"][i] = np.float32(1.0 / 255.0)  # threshold log(1) = 0
    final = O.aaa_cull_remainder(pre, int(d["width"]), int(d["height"]))
    assert final["radii"][i] == 0 and not final["valid"][i] and final["tiles"][i] == 0
    assert final["radii"][other] == pre["radii"][other] and final["valid"][other]


def test_duplicate_pads_a_short_range():
    """The emission's padding (aaa/binning_native.py:76-81), which the golden
    scene does not reach: a Gaussian given more key slots than it has tiles
    fills the rest with tile 0xffffffff, depth FLT_MAX and id -1, and the
    other Gaussians' keys only shift."""
    d = np.load(os.path.join(HERE, "golden", "aaa_coop.npz"))
    pre = _run(d)
    radii, tiles = d["final_radii"], d["final_tiles"].copy()
    i = int(np.flatnonzero(radii > 0)[3])
    tiles[i] += 2
    offsets, keys, values = O.aaa_duplicate(pre, radii, tiles, int(d["width"]), int(d["height"]))
    pad = keys[offsets[i] - 2:offsets[i]]
    assert np.all(values[offsets[i] - 2:offsets[i]] == -1)
    assert np.all(pad >> np.uint64(32) == np.uint64(0xffffffff))
    assert np.all((pad & np.uint64(0xffffffff)) == np.uint64(0x7f7fffff))
    real = values >= 0
    np.testing.assert_array_equal(keys[real], d["dup_keys"])


@pytest.mark.parametrize("path", CASES, ids=lambda p: os.path.basename(p)[:-4])
def test_preprocess_adjoint_matches_reference_kernel(path):
    d = np.load(path)
    ewa = bool(dict(zip(O.AAA_FLAGS, d["flags"].tolist()))["ewa"])
    out = O.aaa_preprocess_backward(
        d["means"], d["quats"], d["scales"], d["opacities"], d["radii"], d["view"], d["proj"],
        d["campos"], int(d["width"]), int(d["height"]), d["adj_focal_x"],
        d["adj_up_transforms"], d["adj_up_opacity"], ewa=ewa)
    for key in ("opacity", "means", "scales", "quats"):
        np.testing.assert_array_equal(out[key], d["adj_" + key], err_msg=key)
    visible = d["radii"] > 0
    assert np.abs(d["adj_quats"][visible]).sum() > 0
    assert not d["adj_means"][~visible].any()


@pytest.mark.parametrize("path", CASES, ids=lambda p: os.path.basename(p)[:-4])
def test_camera_adjoint_matches_reference_kernel(path):
    d = np.load(path)
    use_sh = bool(d["use_sh"])
    rows = O.aaa_camera_backward(
        d["means"], d["quats"], d["scales"], d["radii"], d["opacity"], d["view"], d["proj"],
        d["campos"], int(d["width"]), int(d["height"]), d["cam_focal"], d["adj_up_transforms"],
        d["adj_up_opacity"], d["cam_up_colors"],
        filters=d["filters"] if bool(d["has_filter"]) else None,
        sh=d["sh"] if use_sh else None, sh_degree=int(d["sh_degree"]),
        clamped=d["clamped"] if use_sh else None,
        ewa=bool(dict(zip(O.AAA_FLAGS, d["flags"].tolist()))["ewa"]))
    np.testing.assert_array_equal(rows, d["cam_rows"])
    visible = d["radii"] > 0
    ewa = bool(dict(zip(O.AAA_FLAGS, d["flags"].tolist()))["ewa"])
    assert np.abs(d["cam_rows"][visible][:, :20]).sum() > 0
    # the camera position only receives gradient through the EWA
    # compensation and the SH view direction
    camera_terms = np.abs(d["cam_rows"][visible][:, 20:]).sum()
    assert (camera_terms > 0) == (ewa or use_sh)
    assert not d["cam_rows"][~visible].any()
