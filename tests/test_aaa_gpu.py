"""The AAA-Gaussians sm_100a kernels (through the C ABI) against golden
vectors from dsl_splat's own aaa kernels and against the CPU oracle.

* preprocessing (aaa/preprocess3d.py), the cooperative remainder cull
  (aaa/cooperative_culling.py) and the key emission (aaa/binning_native.py)
  against tests/golden/aaa_*.npz: radii, tile counts, valid flags, queue,
  every projected float and every key bit-exact (atan2, tan, exp and log
  are the library's own functions on both sides);
* the HIER 64/8/4 blend (aaa/render_hierarchical_warp.py) against
  tests/golden/aaa_render_*.npz: image, final transmittance and evaluated
  counts bit-exact; the replay backward's gradients within 1e-3 relative L2
  (float32 atomics in a different order);
* the preprocessing and camera adjoints against the goldens (1e-3 relative
  L2: the golden's exact values, the GPU's atomic sums);
* aaa.rasterize end to end (preprocess, binning, blend, replay, adjoints and
  the pose lowering) against the oracle's composition.
"""

import glob
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import ROOT, rel_l2
from dsl_splat_b200 import aaa
from dsl_splat_b200._native import check, lib
from dsl_splat_b200.aaa import stages as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(ROOT, "tests", "golden")
PRE_CASES = sorted(p for p in glob.glob(os.path.join(GOLDEN, "aaa_*.npz"))
                   if not os.path.basename(p).startswith("aaa_render_"))
RENDER_CASES = sorted(glob.glob(os.path.join(GOLDEN, "aaa_render_*.npz")))
GRAD_TOL = 1e-3


def _dev():
    return torch.device("cuda", 0)


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(_dev())
    return t if dtype is None else t.to(dtype)


def _load(path):
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def _view(d):
    W, H = int(d["width"]), int(d["height"])
    tan = d["tanfov"]
    return S.AaaView(W, H, float(tan[0]), float(tan[1]), tuple(float(v) for v in d["principal"]),
                     _t(d["view"]), _t(d["proj"]), _t(d["campos"]))


def _preprocess_gpu(d):
    """preprocess_3d with the golden's raw flags, through the C ABI."""
    flags = dict(zip(O.AAA_FLAGS, d["flags"].tolist()))
    n = len(d["means"])
    use_sh = bool(d["use_sh"])
    pin = S.Args()
    sh = _t(d["sh"]) if use_sh else None
    f = S.frame(_view(d), aaa.default_settings(), _t(d["means"]), _t(d["quats"]),
                _t(d["scales"]), _t(d["opacities"]),
                _t(d["filters"]) if bool(d["has_filter"]) else None, pin, sh=sh,
                sh_degree=int(d["sh_degree"]), flags=flags)
    dev = _dev()
    out = dict(centers=torch.zeros(n, 2, device=dev), rects=torch.zeros(n, 2, device=dev),
               depths=torch.zeros(n, device=dev), transforms=torch.zeros(n, 4, 4, device=dev),
               opacity=torch.zeros(n, device=dev),
               radii=torch.full((n,), -7, dtype=torch.int32, device=dev),
               tiles=torch.full((n,), -7, dtype=torch.int32, device=dev),
               valid=torch.full((n,), 7, dtype=torch.uint8, device=dev),
               rgb=torch.zeros(n, 3, device=dev), clamped=torch.zeros(n, 3, dtype=torch.uint8,
                                                                        device=dev))
    queued = torch.full((n,), -1, dtype=torch.int32, device=dev)
    size = torch.full((1,), 99, dtype=torch.int32, device=dev)
    s = torch.cuda.current_stream(dev).cuda_stream
    check(lib.splat_aaa_preprocess(
        S.ctypes_ref(f), *(out[k].data_ptr() for k in ("centers", "rects", "depths",
                                                         "transforms", "opacity", "radii",
                                                         "tiles")),
        out["rgb"].data_ptr() if use_sh else None, out["valid"].data_ptr(),
        out["clamped"].data_ptr() if use_sh else None, queued.data_ptr(), size.data_ptr(), s),
          "aaa_preprocess")
    return out, queued, size, f, pin


@pytest.fixture(params=PRE_CASES, ids=[os.path.basename(p)[4:-4] for p in PRE_CASES])
def pre_golden(request):
    return _load(request.param)


def test_preprocess_matches_reference_kernel(pre_golden):
    d = pre_golden
    out, queued, size, f, _ = _preprocess_gpu(d)
    got = {k: v.cpu().numpy() for k, v in out.items()}
    np.testing.assert_array_equal(got["radii"], d["radii"])
    np.testing.assert_array_equal(got["tiles"], d["tiles"])
    np.testing.assert_array_equal(got["valid"].astype(bool), d["valid"])
    q = np.sort(queued[: int(size)].cpu().numpy())
    np.testing.assert_array_equal(q, d["queued"])
    vis = d["radii"] > 0
    assert vis.any()
    for key in ("centers", "rects", "depths", "transforms", "opacity"):
        np.testing.assert_array_equal(got[key][vis], d[key][vis], err_msg=key)
    if bool(d["use_sh"]):
        np.testing.assert_array_equal(got["rgb"][vis], d["rgb"][vis])
        np.testing.assert_array_equal(got["clamped"][vis].astype(bool), d["clamped"][vis])
    if "final_radii" in d:
        s = torch.cuda.current_stream(_dev()).cuda_stream
        check(lib.splat_aaa_cull_remainder(
            len(d["means"]), queued.data_ptr(), size.data_ptr(), out["centers"].data_ptr(),
            out["rects"].data_ptr(), out["transforms"].data_ptr(), out["opacity"].data_ptr(),
            int(d["width"]), int(d["height"]), out["radii"].data_ptr(), out["tiles"].data_ptr(),
            out["valid"].data_ptr(), s), "aaa_cull_remainder")
        for key in ("radii", "tiles"):
            np.testing.assert_array_equal(out[key].cpu().numpy(), d["final_" + key])
        np.testing.assert_array_equal(out["valid"].cpu().numpy().astype(bool), d["final_valid"])


def _emit(d, radii, tiles, centers, rects, transforms, opacity, offsets=None):
    W, H = int(d["width"]), int(d["height"])
    n = len(radii)
    if offsets is None:
        offsets = np.cumsum(np.where(radii > 0, tiles, 0)).astype(np.int32)
    m = int(offsets[-1])
    t_out = torch.full((m,), 7, dtype=torch.int32, device=_dev())
    d_out = torch.full((m,), 7, dtype=torch.int32, device=_dev())
    i_out = torch.full((m,), -7, dtype=torch.int32, device=_dev())
    s = torch.cuda.current_stream(_dev()).cuda_stream
    offsets_d, radii_d = _t(offsets), _t(radii)  # referenced until the kernel ran
    check(lib.splat_aaa_emit(n, m, offsets_d.data_ptr(), centers.data_ptr(), rects.data_ptr(),
                             radii_d.data_ptr(), transforms.data_ptr(), opacity.data_ptr(), W,
                             H, t_out.data_ptr(), d_out.data_ptr(), i_out.data_ptr(), s),
          "aaa_emit")
    torch.cuda.synchronize(_dev())
    T = ((W + 15) // 16) * ((H + 15) // 16)
    pad = (1 << T.bit_length()) - 1
    tiles_np = t_out.cpu().numpy().view(np.uint32).astype(np.uint64)
    depth_bits = d_out.cpu().numpy().view(np.uint32).astype(np.uint64) + np.uint64(0x40E00000)
    ids = i_out.cpu().numpy()
    keys = (tiles_np << np.uint64(32)) | depth_bits
    padding = ids == -1
    keys[padding] = (np.uint64(0xffffffff) << np.uint64(32)) | np.uint64(0x7f7fffff)
    assert np.all(tiles_np[padding] == pad)
    return offsets, keys, ids


def test_emission_and_binning_match_reference_kernel():
    d = _load(os.path.join(GOLDEN, "aaa_coop.npz"))
    out, queued, size, _, _ = _preprocess_gpu(d)
    W, H = int(d["width"]), int(d["height"])
    args = [_t(d[k]) for k in ("centers", "rects", "transforms", "opacity")]
    offsets, keys, ids = _emit(d, d["final_radii"], d["final_tiles"], *args)
    np.testing.assert_array_equal(offsets, d["dup_offsets"])
    np.testing.assert_array_equal(keys, d["dup_keys"])
    np.testing.assert_array_equal(ids, d["dup_values"])
    # the sort and ranges (primitives/tiling.py:39-100) against the oracle's
    # stable sort of the reference keys
    T = ((W + 15) // 16) * ((H + 15) // 16)
    _, want_ids, want_ranges = O.aaa_sort(d["dup_keys"], d["dup_values"], T)
    m = len(want_ids)
    ws = torch.empty(lib.splat_aaa_bin_workspace_bytes(m), dtype=torch.uint8, device=_dev())
    point_list = torch.empty(m, dtype=torch.int32, device=_dev())
    ranges = torch.full((T, 2), 7, dtype=torch.int32, device=_dev())
    s = torch.cuda.current_stream(_dev()).cuda_stream
    offsets_d, radii_d = _t(offsets), _t(d["final_radii"])
    check(lib.splat_aaa_bin(len(d["means"]), m, offsets_d.data_ptr(), args[0].data_ptr(),
                            args[1].data_ptr(), radii_d.data_ptr(), args[2].data_ptr(),
                            args[3].data_ptr(), W, H, ws.data_ptr(), ws.numel(),
                            point_list.data_ptr(), ranges.data_ptr(), s), "aaa_bin")
    torch.cuda.synchronize(_dev())
    np.testing.assert_array_equal(point_list.cpu().numpy(), want_ids)
    np.testing.assert_array_equal(ranges.cpu().numpy(), want_ranges)


def test_emission_pads_a_short_range():
    """A Gaussian given more key slots than it has tiles fills the rest with
    padding (aaa/binning_native.py:76-81); the other pairs only shift."""
    d = _load(os.path.join(GOLDEN, "aaa_coop.npz"))
    radii, tiles = d["final_radii"], d["final_tiles"].copy()
    i = int(np.flatnonzero(radii > 0)[3])
    tiles[i] += 2
    args = [_t(d[k]) for k in ("centers", "rects", "transforms", "opacity")]
    offsets, keys, ids = _emit(d, radii, tiles, *args)
    assert np.all(ids[offsets[i] - 2:offsets[i]] == -1)
    np.testing.assert_array_equal(keys[ids >= 0], d["dup_keys"])


def test_binning_at_scale_against_oracle():
    """Emission, sort and ranges of a 60k-Gaussian view (many long
    rectangles, deep tiles) against the oracle, bit for bit."""
    from dsl_splat_b200.scenes import make_scene
    sc = make_scene(1, n=60000, width=640, height=360)
    cams = aaa.cameras.prepare_cameras(sc.viewmats[None].to(_dev()), sc.Ks[None].to(_dev()),
                                       sc.width, sc.height, 0.01, 1e10)
    view = cams.view(0, 0)
    q = F.normalize(sc.quats.to(_dev()), dim=-1)
    st = S.preprocess(view, aaa.default_settings(), sc.means.to(_dev()), q,
                      sc.scales.to(_dev()), sc.opacities.to(_dev()))
    bins, _ = S.bin_and_sort_many([st], sc.width, sc.height)
    pre = O.aaa_preprocess(sc.means.numpy(), q.cpu().numpy(), sc.scales.numpy(),
                           sc.opacities.numpy(), view.viewmatrix.cpu().numpy(),
                           view.projmatrix.cpu().numpy(), view.campos.cpu().numpy(), sc.width,
                           sc.height, (view.tanfovx, view.tanfovy), view.principal)
    final = O.aaa_cull_remainder(pre, sc.width, sc.height)
    np.testing.assert_array_equal(st.radii.cpu().numpy(), final["radii"])
    np.testing.assert_array_equal(st.tiles.cpu().numpy(), final["tiles"])
    _, keys, values = O.aaa_duplicate(pre, final["radii"], final["tiles"], sc.width, sc.height)
    T = ((sc.width + 15) // 16) * ((sc.height + 15) // 16)
    _, ids, ranges = O.aaa_sort(keys, values, T)
    assert len(ids) > 100000
    np.testing.assert_array_equal(bins[0]["point_list"].cpu().numpy(), ids)
    np.testing.assert_array_equal(bins[0]["ranges"].cpu().numpy(), ranges)


@pytest.fixture(params=RENDER_CASES, ids=[os.path.basename(p)[11:-4] for p in RENDER_CASES])
def render_golden(request):
    return _load(request.param)


def _render_inputs(g):
    st = S.AaaState(None, None, None, _t(g["transforms"]), _t(g["opacity"]), None, None, None)
    bins = dict(ranges=_t(g["ranges"]), point_list=_t(g["ids"]))
    return st, bins


def test_hier_blend_matches_reference_kernel(render_golden):
    g = render_golden
    W, H = int(g["width"]), int(g["height"])
    st, bins = _render_inputs(g)
    for order in (None, "heaviest first"):
        if order:
            from dsl_splat_b200 import stages as core
            bins["tile_order"] = core.tile_order(dict(ranges=bins["ranges"]))
        image, final_t, contrib, _ = S.render(st, bins, _t(g["features"]), _t(g["background"]),
                                              W, H, bool(g["cull"]))
        np.testing.assert_array_equal(contrib.cpu().numpy(), g["contributors"])
        np.testing.assert_array_equal(final_t.cpu().numpy(), g["final_t"])
        np.testing.assert_array_equal(image.cpu().numpy(), g["image"])


def test_hier_statistics_match_reference_kernel(render_golden):
    """The statistics variant of the blend (render_statistics): the image is
    unchanged, the masked count bit for bit, the weighted sum within 1e-5
    relative L2 (float32 atomics in a different order)."""
    from dsl_splat_b200.statistics import PreparedStatistics
    g = render_golden
    if "stat_counts" not in g:
        pytest.skip("this golden has no statistics requests")
    W, H = int(g["width"]), int(g["height"])
    st, bins = _render_inputs(g)
    n = len(g["opacity"])
    maps = _t(np.stack([g["stat_mask"].ravel(), g["stat_weights"].ravel()]))
    stats = PreparedStatistics((0, 1), maps, torch.zeros((1, n), device=_dev(), dtype=torch.int32),
                               torch.zeros((1, n), device=_dev()))
    image, _, _, _ = S.render(st, bins, _t(g["features"]), _t(g["background"]), W, H,
                              bool(g["cull"]), statistics=stats)
    np.testing.assert_array_equal(image.cpu().numpy(), g["image"])
    np.testing.assert_array_equal(stats.counts[0].cpu().numpy(), g["stat_counts"])
    assert rel_l2(stats.sums[0].cpu(), g["stat_sums"]) <= 1e-5


def test_hier_replay_matches_reference_kernel(render_golden):
    g = render_golden
    W, H = int(g["width"]), int(g["height"])
    st, bins = _render_inputs(g)
    for screen, absgrad in ((False, False), (True, False), (True, True)):
        g_tr, g_op, g_col, g_scr, g_abs = S.render_backward(
            st, bins, _t(g["features"]), _t(g["background"]), _t(g["image"]), _t(g["final_t"]),
            _t(g["upstream"]), W, H, bool(g["cull"]), screen=screen, absgrad=absgrad)
        assert rel_l2(g_tr.reshape(-1, 16).cpu(), g["grad_transforms"]) <= GRAD_TOL
        assert rel_l2(g_op.cpu(), g["grad_opacity"]) <= GRAD_TOL
        assert rel_l2(g_col.cpu(), g["grad_features"]) <= GRAD_TOL
        if screen:
            assert rel_l2(g_scr.cpu(), g["grad_screen"]) <= GRAD_TOL
        if absgrad:
            assert rel_l2(g_abs.cpu(), g["grad_screen_abs"]) <= GRAD_TOL


@pytest.mark.parametrize("capacity", [256, 3])
def test_recorded_backward_matches_reference_kernel(render_golden, capacity):
    """The backward from the forward's blend records: capacity 256 records
    every pixel of the golden scenes; capacity 3 overflows most tiles, which the replay
    kernel then handles while the others use their records.  Both must give
    the reference replay's gradients, and the forward is unchanged by
    recording."""
    g = render_golden
    W, H = int(g["width"]), int(g["height"])
    st, bins = _render_inputs(g)
    feats, bg = _t(g["features"]), _t(g["background"])
    image, final_t, contrib, rec = S.render(st, bins, feats, bg, W, H, bool(g["cull"]),
                                            record_capacity=capacity)
    np.testing.assert_array_equal(image.cpu().numpy(), g["image"])
    np.testing.assert_array_equal(contrib.cpu().numpy(), g["contributors"])
    overflowed = int(rec["overflow"].sum())
    if capacity == 256:
        assert overflowed == 0
    else:
        assert 0 < overflowed < len(rec["overflow"]) or overflowed == len(rec["overflow"])
    counts = rec["counts"].cpu().numpy()
    assert counts.max() <= capacity and (counts == -1).any() == (capacity == 3)
    g_tr, g_op, g_col, g_scr, g_abs = S.render_backward(
        st, bins, feats, bg, image, final_t, _t(g["upstream"]), W, H, bool(g["cull"]),
        screen=True, absgrad=True, records=rec)
    assert rel_l2(g_tr.reshape(-1, 16).cpu(), g["grad_transforms"]) <= GRAD_TOL
    assert rel_l2(g_op.cpu(), g["grad_opacity"]) <= GRAD_TOL
    assert rel_l2(g_col.cpu(), g["grad_features"]) <= GRAD_TOL
    assert rel_l2(g_scr.cpu(), g["grad_screen"]) <= GRAD_TOL
    assert rel_l2(g_abs.cpu(), g["grad_screen_abs"]) <= GRAD_TOL


def test_preprocess_and_camera_adjoints_match_reference_kernels(pre_golden):
    d = pre_golden
    flags = dict(zip(O.AAA_FLAGS, d["flags"].tolist()))
    view = _view(d)
    st = S.AaaState(None, None, None, None, _t(d["opacity"]), _t(d["radii"]), None, None)
    up_t, up_o = _t(d["adj_up_transforms"]), _t(d["adj_up_opacity"])
    settings = aaa.default_settings(antialiased=bool(flags["ewa"]))
    n = len(d["means"])
    s = torch.cuda.current_stream(_dev()).cuda_stream
    pin = S.Args()
    f = S.frame(view, settings, _t(d["means"]), _t(d["quats"]), _t(d["scales"]),
                _t(d["opacities"]), None, pin, flags=flags)
    f.focal_x = float(d["adj_focal_x"])  # the reference's float32 kernel argument
    outs = [torch.full((n,) + shape, 7.0, device=_dev()) for shape in ((), (3,), (3,), (4,))]
    check(lib.splat_aaa_preprocess_backward(S.ctypes_ref(f), st.radii.data_ptr(), up_t.data_ptr(),
                                            up_o.data_ptr(), *(o.data_ptr() for o in outs), s),
          "aaa_preprocess_backward")
    # per-Gaussian arithmetic in the reference's order, no atomics
    for got, key in zip(outs, ("opacity", "means", "scales", "quats")):
        assert rel_l2(got.cpu(), d["adj_" + key]) <= 1e-6, key
    if bool(d["use_sh"]):
        return  # the camera adjoint's SH term is computed by the SH stage on this path
    f = S.frame(view, settings, _t(d["means"]), _t(d["quats"]), _t(d["scales"]), _t(d["opacity"]),
                _t(d["filters"]) if bool(d["has_filter"]) else None, pin, flags=flags)
    f.focal_max = float(d["cam_focal"])
    sums = torch.empty(23, device=_dev())
    radii_d, opacity_d = _t(d["radii"]), _t(d["opacity"])
    check(lib.splat_aaa_camera_backward(S.ctypes_ref(f), radii_d.data_ptr(),
                                        opacity_d.data_ptr(), up_t.data_ptr(),
                                        up_o.data_ptr(), sums.data_ptr(), s),
          "aaa_camera_backward")
    want = d["cam_rows"].astype(np.float64).sum(0)
    assert rel_l2(sums.cpu()[:20], want[:20]) <= 1e-5
    if flags["ewa"]:
        assert rel_l2(sums.cpu()[20:], want[20:]) <= 1e-5
    else:
        assert not sums[20:].any()


def _oracle_aaa(sc, q_np, view, features, bg, gF):
    """The oracle's composition of one aaa.rasterize view: preprocessing,
    remainder cull, emission, sort, HIER blend, replay, both adjoints."""
    W, H = sc.width, sc.height
    args = (view.viewmatrix.cpu().numpy(), view.projmatrix.cpu().numpy(),
            view.campos.cpu().numpy())
    pre = O.aaa_preprocess(sc.means.numpy(), q_np, sc.scales.numpy(), sc.opacities.numpy(), *args,
                           W, H, (view.tanfovx, view.tanfovy), view.principal)
    final = O.aaa_cull_remainder(pre, W, H)
    _, keys, values = O.aaa_duplicate(pre, final["radii"], final["tiles"], W, H)
    T = ((W + 15) // 16) * ((H + 15) // 16)
    _, ids, ranges = O.aaa_sort(keys, values, T)
    image, final_t, contrib = O.aaa_render(W, H, ranges, ids, pre["transforms"], pre["opacity"],
                                           features, bg)
    g = O.aaa_render_backward(W, H, ranges, ids, pre["transforms"], pre["opacity"], features, bg,
                              image, final_t, gF, screen=True, absgrad=True)
    up_t = g["transforms"].astype(np.float32)
    up_o = g["opacity"].astype(np.float32)
    adj = O.aaa_preprocess_backward(sc.means.numpy(), q_np, sc.scales.numpy(),
                                    sc.opacities.numpy(), final["radii"], *args, W, H,
                                    np.float32(W / (2.0 * view.tanfovx)), up_t, up_o)
    rows = O.aaa_camera_backward(sc.means.numpy(), q_np, sc.scales.numpy(), final["radii"],
                                 pre["opacity"], *args, W, H,
                                 np.float32(max(W / (2 * view.tanfovx), H / (2 * view.tanfovy))),
                                 up_t, up_o, np.zeros(3 * len(q_np), np.float32))
    return dict(pre=pre, final=final, image=image, final_t=final_t, contrib=contrib, grads=g,
                adj=adj, camera=rows.astype(np.float64).sum(0))


def test_rasterize_matches_oracle():
    """aaa.rasterize (features + 2 extras over a background) forward and
    backward against the oracle composition: images bit-exact; gradients of
    means, quaternions (through F.normalize), scales, opacities, features,
    extras, means2d / absgrad and the pose within 1e-3 relative L2."""
    from dsl_splat_b200.scenes import make_scene
    dev = _dev()
    sc = make_scene(1, n=20000, width=480, height=272)
    gen = torch.Generator().manual_seed(31)
    colors = torch.rand(sc.means.shape[0], 3, generator=gen)
    extras = torch.randn(sc.means.shape[0], 2, generator=gen)
    bg = torch.tensor([0.2, 0.4, 0.6])
    leaves = {k: getattr(sc, k).to(dev).requires_grad_(True)
              for k in ("means", "quats", "scales", "opacities")}
    feats = colors.to(dev).requires_grad_(True)
    ex = extras.to(dev).requires_grad_(True)
    vm = sc.viewmats.to(dev).requires_grad_(True)
    res = aaa.rasterize(leaves["means"], leaves["quats"], leaves["scales"], leaves["opacities"],
                        vm, sc.Ks.to(dev), sc.width, sc.height, features=feats,
                        extra_features=ex, backgrounds=bg.to(dev)[None], absgrad=True)
    H, W = sc.height, sc.width
    gF = torch.randn(1, H, W, 3, generator=gen)
    gE = torch.randn(1, H, W, 2, generator=gen)
    gA = torch.randn(1, H, W, 1, generator=gen)
    ((res.features * gF.to(dev)).sum() + (res.extra_features * gE.to(dev)).sum()
     + (res.alpha * gA.to(dev)).sum()).backward()

    cams = aaa.cameras.prepare_cameras(sc.viewmats[None].to(dev), sc.Ks[None].to(dev), W, H,
                                       0.01, 1e10)
    view = cams.view(0, 0)
    qn = F.normalize(sc.quats.to(dev), dim=-1).cpu()
    features = np.concatenate([colors.numpy(), extras.numpy(), np.ones((len(colors), 1))], 1)
    bg_full = np.array([0.2, 0.4, 0.6, 0.0, 0.0, 0.0], np.float32)
    up = np.concatenate([gF[0].numpy(), gE[0].numpy(), gA[0].numpy()], -1)
    want = _oracle_aaa(sc, qn.numpy(), view, features.astype(np.float32), bg_full,
                       np.moveaxis(up, -1, 0).copy())
    got = torch.cat([res.features, res.extra_features, res.alpha], -1)[0].detach().cpu().numpy()
    np.testing.assert_array_equal(np.moveaxis(got, -1, 0), want["image"])
    np.testing.assert_array_equal((res.radii[0] > 0).any(-1).cpu().numpy(),
                                  want["final"]["radii"] > 0)
    g = want["grads"]
    assert rel_l2(feats.grad.cpu(), g["colors"][:, :3]) <= GRAD_TOL
    assert rel_l2(ex.grad.cpu(), g["colors"][:, 3:5]) <= GRAD_TOL
    assert rel_l2(res.means2d.grad[0].cpu(), g["screen"]) <= GRAD_TOL
    assert rel_l2(res.means2d.absgrad[0].cpu(), g["screen_abs"]) <= GRAD_TOL
    adj = want["adj"]
    assert rel_l2(leaves["means"].grad.cpu(), adj["means"]) <= GRAD_TOL
    assert rel_l2(leaves["scales"].grad.cpu(), adj["scales"]) <= GRAD_TOL
    assert rel_l2(leaves["opacities"].grad.cpu(), adj["opacity"]) <= GRAD_TOL
    _, vjp = torch.func.vjp(lambda x: F.normalize(x, dim=-1), sc.quats.double())
    gq = vjp(torch.from_numpy(adj["quats"].astype(np.float64)))[0].numpy()
    assert rel_l2(leaves["quats"].grad.cpu(), gq) <= GRAD_TOL
    # the pose: the camera adjoint's sums carried through the Torch lowering
    vm2 = sc.viewmats[None].to(dev).clone().requires_grad_(True)
    low = aaa.cameras.prepare_cameras(vm2, sc.Ks[None].to(dev), W, H, 0.01, 1e10)
    s = torch.from_numpy(want["camera"]).float().to(dev)
    g_view = torch.zeros(4, 4, device=dev)
    g_view[:, 2] = s[16:20]
    torch.autograd.backward([low.projection[0, 0], low.transposed_views[0, 0],
                             low.centers[0, 0]], [s[:16].view(4, 4), g_view, s[20:23]])
    assert rel_l2(vm.grad.cpu(), vm2.grad[0].cpu()) <= GRAD_TOL


def test_rasterize_sh_and_gsplat_adapter():
    """SH colours go through the SH stage (colours = SH at means - camera
    centre, exactly what features= receives), and the gsplat adapter returns
    the same images; packed metadata lists the visible Gaussians."""
    from dsl_splat_b200.scenes import make_scene
    dev = _dev()
    sc = make_scene(1, n=8000, width=320, height=192)
    args = [getattr(sc, k).to(dev) for k in ("means", "quats", "scales", "opacities")]
    vm, Ks = sc.viewmats.to(dev), sc.Ks.to(dev)
    sh = sc.sh_coeffs.to(dev)
    res = aaa.rasterize(*args, vm, Ks, sc.width, sc.height, sh_coeffs=sh)
    from dsl_splat_b200.inputs import spherical_harmonics
    cams = aaa.cameras.prepare_cameras(vm[None], Ks[None], sc.width, sc.height, 0.01, 1e10)
    colors = spherical_harmonics(sh, args[0] - cams.centers[0, 0], 3)
    res2 = aaa.rasterize(*args, vm, Ks, sc.width, sc.height, features=colors)
    assert torch.equal(res.features, res2.features)
    assert torch.equal(res.alpha, res2.alpha)
    feats, alpha, meta = aaa.gsplat.rasterization(*args, sh, vm, Ks, sc.width, sc.height,
                                                  sh_degree=3, packed=True,
                                                  rasterize_mode="antialiased")
    assert torch.equal(feats, res.features) and torch.equal(alpha, res.alpha)
    vis = (res.radii[0] > 0).all(-1)
    assert meta["packed"] is True and len(meta["means2d"]) == int(vis.sum())
    with pytest.raises(NotImplementedError):
        aaa.gsplat.rasterization(*args, sh, vm, Ks, sc.width, sc.height, sh_degree=3,
                                 with_eval3d=False)


@pytest.mark.parametrize("case", ["empty", "behind_camera"])
def test_rasterize_empty_and_culled(case):
    from dsl_splat_b200.scenes import make_scene
    dev = _dev()
    sc = make_scene(0, n=0 if case == "empty" else 300)
    means = sc.means.to(dev)
    if case == "behind_camera":
        means = means * torch.tensor([1.0, 1.0, -1.0], device=dev)
    bg = torch.tensor([[0.3, 0.2, 0.1]], device=dev)
    res = aaa.rasterize(means, sc.quats.to(dev), sc.scales.to(dev), sc.opacities.to(dev),
                        sc.viewmats.to(dev), sc.Ks.to(dev), sc.width, sc.height,
                        sh_coeffs=sc.sh_coeffs.to(dev), backgrounds=bg)
    want = bg.view(1, 1, 1, 3).expand(1, sc.height, sc.width, 3)
    assert torch.equal(res.features, want)
    assert not res.alpha.any()


def test_recorded_backward_dense_tile_takes_the_per_sample_path():
    """A tile whose blended samples exceed the record backward's per-tile list
    (24,576 samples) is reduced sample by sample; its gradients equal the
    replay's, and a second backward of the same records replays."""
    dev = _dev()
    n, W, H = 200, 64, 64
    gen = torch.Generator().manual_seed(5)
    means = torch.cat([torch.randn(n, 2, generator=gen) * 0.05,
                       4.0 + torch.rand(n, 1, generator=gen)], 1)
    quats = F.normalize(torch.randn(n, 4, generator=gen), dim=-1)
    scales = torch.full((n, 3), 2.0)
    opacities = torch.full((n,), 0.01)
    K = torch.tensor([[100.0, 0.0, 32.0], [0.0, 100.0, 32.0], [0.0, 0.0, 1.0]])
    cams = aaa.cameras.prepare_cameras(torch.eye(4)[None, None].to(dev), K[None, None].to(dev),
                                       W, H, 0.01, 1e10)
    st = S.preprocess(cams.view(0, 0), aaa.default_settings(), means.to(dev), quats.to(dev),
                      scales.to(dev), opacities.to(dev))
    bins, _ = S.bin_and_sort_many([st], W, H)
    feats = torch.rand(n, 4, generator=gen).to(dev)
    feats[:, 3] = 1.0
    bg = torch.zeros(4, device=dev)
    image, final_t, _, rec = S.render(st, bins[0], feats, bg, W, H, True, record_capacity=256)
    assert int(rec["overflow"].sum()) == 0
    assert int(rec["counts"].view(-1, 256).sum(1).max()) > 24576
    up = torch.randn(4, H, W, generator=gen).to(dev)
    args = (st, bins[0], feats, bg, image, final_t, up, W, H, True)
    got = S.render_backward(*args, screen=True, absgrad=True, records=rec)
    assert rec["consumed"]
    again = S.render_backward(*args, screen=True, absgrad=True, records=rec)
    want = S.render_backward(*args, screen=True, absgrad=True)
    for a, b, c in zip(got, want, again):
        assert rel_l2(a.cpu(), b.cpu()) <= 1e-4
        assert torch.equal(b, c) or rel_l2(c.cpu(), b.cpu()) <= 1e-5


def test_rasterize_statistics_against_oracle():
    """aaa.rasterize with a masked count and a weighted sum over two cameras
    (statistics.py's requests, owned (C, N) outputs) against the oracle's
    observer on each view: counts bit for bit, sums within 1e-5."""
    from dsl_splat_b200.scenes import make_scene
    from dsl_splat_b200.statistics import MaskedContributionCount, WeightedContributionSum
    dev = _dev()
    sc = make_scene(1, n=6000, width=160, height=96)
    gen = torch.Generator().manual_seed(41)
    colors = torch.rand(sc.means.shape[0], 3, generator=gen)
    H, W = sc.height, sc.width
    mask = torch.rand(H, W, generator=gen) > 0.5
    weights = torch.rand(2, H, W, generator=gen)
    vms = torch.cat([sc.viewmats[:1], sc.viewmats[:1].clone()])  # (2, 4, 4)
    vms[1, 0, 3] += 0.05
    Ks = torch.cat([sc.Ks[:1], sc.Ks[:1]])
    args = [getattr(sc, k).to(dev) for k in ("means", "quats", "scales", "opacities")]
    res = aaa.rasterize(*args, vms.to(dev), Ks.to(dev), W, H, features=colors.to(dev),
                        statistics=(MaskedContributionCount("hits", mask.to(dev)),
                                    WeightedContributionSum("weight", weights.to(dev))))
    assert set(res.statistics) == {"hits", "weight"}
    assert res.statistics["hits"].shape == (2, len(colors))
    qn = F.normalize(sc.quats.to(dev), dim=-1).cpu().numpy()  # CUDA F.normalize bits
    cams = aaa.cameras.prepare_cameras(vms.to(dev)[None], Ks.to(dev)[None], W, H, 0.01, 1e10)
    features = np.concatenate([colors.numpy(), np.ones((len(colors), 1))], 1).astype(np.float32)
    for c in range(2):
        view = cams.view(0, c)
        vargs = (view.viewmatrix.cpu().numpy(), view.projmatrix.cpu().numpy(),
                 view.campos.cpu().numpy())
        pre = O.aaa_preprocess(sc.means.numpy(), qn, sc.scales.numpy(), sc.opacities.numpy(),
                               *vargs, W, H, (view.tanfovx, view.tanfovy), view.principal)
        final = O.aaa_cull_remainder(pre, W, H)
        _, keys, values = O.aaa_duplicate(pre, final["radii"], final["tiles"], W, H)
        T = ((W + 15) // 16) * ((H + 15) // 16)
        _, ids, ranges = O.aaa_sort(keys, values, T)
        maps = np.stack([mask.numpy().astype(np.float32), weights[c].numpy()])
        _, _, _, counts, sums = O.aaa_render(W, H, ranges, ids, pre["transforms"],
                                             pre["opacity"], features, np.zeros(4, np.float32),
                                             stat_maps=maps, stat_kinds=(0, 1))
        np.testing.assert_array_equal(res.statistics["hits"][c].cpu().numpy(), counts[0])
        assert counts[0].any()
        assert rel_l2(res.statistics["weight"][c].cpu(), sums[0]) <= 1e-5


@pytest.mark.parametrize("channels", [2, 9, 33])
def test_recorded_backward_wide_features(channels):
    """The record backward's per-channel paths (fewer than four channels,
    and 16- / 64-channel instantiations): gradients equal the replay's on a
    dense view."""
    from dsl_splat_b200.scenes import make_scene
    dev = _dev()
    sc = make_scene(1, n=12000, width=192, height=128)
    cams = aaa.cameras.prepare_cameras(sc.viewmats[None].to(dev), sc.Ks[None].to(dev),
                                       sc.width, sc.height, 0.01, 1e10)
    q = F.normalize(sc.quats.to(dev), dim=-1)
    st = S.preprocess(cams.view(0, 0), aaa.default_settings(), sc.means.to(dev), q,
                      sc.scales.to(dev), sc.opacities.to(dev))
    bins, _ = S.bin_and_sort_many([st], sc.width, sc.height)
    gen = torch.Generator().manual_seed(channels)
    feats = torch.rand(len(q), channels, generator=gen).to(dev)
    bg = torch.rand(channels, generator=gen).to(dev)
    W, H = sc.width, sc.height
    image, final_t, _, rec = S.render(st, bins[0], feats, bg, W, H, True, record_capacity=192)
    plain, plain_t, _, _ = S.render(st, bins[0], feats, bg, W, H, True)
    assert torch.equal(image, plain) and torch.equal(final_t, plain_t)
    assert int(rec["overflow"].sum()) < len(rec["overflow"])
    up = torch.randn(channels, H, W, generator=gen).to(dev)
    args = (st, bins[0], feats, bg, image, final_t, up, W, H, True)
    got = S.render_backward(*args, screen=True, absgrad=True, records=rec)
    want = S.render_backward(*args, screen=True, absgrad=True)
    for a, b in zip(got, want):
        assert b.abs().sum() > 0
        assert rel_l2(a.cpu(), b.cpu()) <= 1e-4


def test_stage_ops_compose_like_rasterize():
    """aaa.ops (aaa/ops.py:320-464): prepare_gaussians -> bin_and_sort ->
    rasterize_to_pixels gives aaa.rasterize's images and statistics bit for
    bit and its gradients (Gaussians, features, pose) within 1e-4."""
    from dsl_splat_b200.cameras import PinholeCamera
    from dsl_splat_b200.scenes import make_scene
    from dsl_splat_b200.statistics import MaskedContributionCount
    dev = _dev()
    sc = make_scene(1, n=8000, width=256, height=160)
    W, H = sc.width, sc.height
    gen = torch.Generator().manual_seed(53)
    colors = torch.rand(len(sc.means), 3, generator=gen).to(dev)
    bg = torch.tensor([0.1, 0.5, 0.9], device=dev)
    mask = (torch.rand(H, W, generator=gen) > 0.3).to(dev)
    gF = torch.randn(H, W, 3, generator=gen).to(dev)
    gA = torch.randn(H, W, 1, generator=gen).to(dev)

    def leaves():
        out = {k: getattr(sc, k).to(dev).requires_grad_(True)
               for k in ("means", "quats", "scales", "opacities")}
        out["features"] = colors.clone().requires_grad_(True)
        out["viewmat"] = sc.viewmats[0].to(dev).requires_grad_(True)
        return out

    a = leaves()
    camera = PinholeCamera(a["viewmat"], sc.Ks[0].to(dev), W, H)
    geo = aaa.ops.prepare_gaussians(a["means"], a["quats"], a["scales"], a["opacities"], camera)
    tiles = aaa.ops.bin_and_sort(geo)
    px = aaa.ops.rasterize_to_pixels(geo, tiles, a["features"], bg,
                                     statistics=(MaskedContributionCount("hits", mask),))
    ((px.features * gF).sum() + (px.alpha * gA).sum()).backward()

    b = leaves()
    res = aaa.rasterize(b["means"], b["quats"], b["scales"], b["opacities"], b["viewmat"][None],
                        sc.Ks[:1].to(dev), W, H, features=b["features"], backgrounds=bg[None],
                        statistics=(MaskedContributionCount("hits", mask),))
    ((res.features[0] * gF).sum() + (res.alpha[0] * gA).sum()).backward()
    assert torch.equal(px.features, res.features[0]) and torch.equal(px.alpha, res.alpha[0])
    assert torch.equal(px.statistics["hits"], res.statistics["hits"][0])
    np.testing.assert_array_equal(geo.radii.cpu().numpy() > 0,
                                  (res.radii[0] > 0).any(-1).cpu().numpy())
    for name in ("means", "quats", "scales", "opacities", "features", "viewmat"):
        assert a[name].grad is not None and a[name].grad.abs().sum() > 0, name
        assert rel_l2(a[name].grad.cpu(), b[name].grad.cpu()) <= 1e-4, name
    with pytest.raises(ValueError):
        aaa.ops.rasterize_to_pixels(geo, aaa.ops.bin_and_sort(geo), a["features"][:, :2][:-1])
