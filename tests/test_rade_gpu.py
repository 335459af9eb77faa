"""The RaDe-GS sm_100a kernels (through the C ABI) against golden vectors
from dsl_splat's own rade kernels and against the CPU oracle.

Tolerances: radii, tile counts, sort keys and ids, ranges and contributors
bit-exact; projection floats bit-exact; images, depths and normals max-abs
1e-5; gradients relative L2 1e-3 (float32 atomics in arbitrary order; the
projection backward against the float64 autograd oracle).
"""

import glob
import os

import numpy as np
import pytest
import torch

from conftest import ROOT, rel_l2
from dsl_splat_b200 import rade, stages
from dsl_splat_b200.rade import projection as rproj
from dsl_splat_b200.rade import render as rrender
from oracle import oracle as O
from oracle import rade_vjp

pytestmark = pytest.mark.gpu

FIXTURES = sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "rade_*.npz")))


@pytest.fixture(params=FIXTURES, ids=[os.path.basename(p)[5:-4] for p in FIXTURES])
def golden(request):
    with np.load(request.param) as z:
        return {k: z[k] for k in z.files}


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")
    return t if dtype is None else t.to(dtype)


def _config(g):
    return rproj.ViewConfig(int(g["width"]), int(g["height"]), 0.2, float("inf"), 0.0, "radius",
                            float(g["kernel_size"]))


def _project(g):
    return rproj.prepare(_t(g["means"]), _t(g["quats"]), _t(g["scales"]), _t(g["opacities"]),
                         _t(g["viewmat"]), _t(g["full"]), _t(g["K"]), _config(g))


def _forward_from_planar(g):
    """The golden forward (planar (C+6,H,W) as the reference stores it) as
    the five channel-last images the B200 blend writes."""
    img = _t(g["image"]).permute(1, 2, 0)
    parts = (img[..., :-6], img[..., -6:-5], img[..., -5:-4], img[..., -4:-3], img[..., -3:])
    return rrender.RenderedPixels(*(t.contiguous() for t in parts), _t(g["auxiliary"]),
                                  _t(g["contributors"]))


def _golden_state(g):
    return rproj.ProjectedGaussians(_t(g["centers"]), _t(g["conics"]), _t(g["radii"]),
                                    _t(g["tiles"]), _t(g["depths"]), _t(g["planes"]),
                                    _t(g["normals"]))


def test_rade_projection_and_bins_match_reference_kernels(golden):
    g = golden
    st = _project(g)
    radii = st.radii.cpu().numpy()
    np.testing.assert_array_equal(radii, g["radii"])
    np.testing.assert_array_equal(st.tile_counts.cpu().numpy(), g["tiles"])
    vis = radii > 0
    for name, t in (("centers", st.centers), ("conics", st.conics), ("depths", st.depths),
                    ("planes", st.ray_planes), ("normals", st.normals)):
        np.testing.assert_array_equal(t.cpu().numpy()[vis], g[name][vis], err_msg=name)
    bins = stages.bin_and_sort(st, int(g["width"]), int(g["height"]))
    np.testing.assert_array_equal(bins["ranges"].cpu().numpy(), g["ranges"])
    np.testing.assert_array_equal(bins["point_list"].cpu().numpy(), g["ids"])


def test_rade_render_matches_reference_kernels(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    st = _golden_state(g)
    bins = dict(ranges=_t(g["ranges"]), point_list=_t(g["ids"]))
    out = rrender.render(st, bins, _t(g["colors"]), _t(g["extras"]) if g["extras"].shape[1] else None,
                         _t(g["background"]), _t(g["K"]), W, H)
    np.testing.assert_array_equal(out.contributors.cpu().numpy(), g["contributors"])
    np.testing.assert_allclose(out.planar().cpu().numpy(), g["image"], rtol=0, atol=1e-5)
    np.testing.assert_allclose(out.auxiliary.cpu().numpy(), g["auxiliary"], rtol=0, atol=1e-5)


def test_rade_render_backward_matches_reference_kernels(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    st = _golden_state(g)
    bins = dict(ranges=_t(g["ranges"]), point_list=_t(g["ids"]))
    extras = _t(g["extras"]) if g["extras"].shape[1] else None
    fwd = _forward_from_planar(g)
    ups = tuple(_t(g[k]) for k in ("up_features", "up_alpha", "up_depth", "up_median",
                                   "up_normals"))
    gc, gq, ga, gb, gp, gn, gabs = rrender.backward(
        st, bins, _t(g["colors"]), extras, _t(g["background"]), _t(g["K"]), fwd, ups, W, H,
        absgrad=True)
    feats = ga if gb is None else torch.cat([ga, gb], 1)
    for got, ref in ((gc, "grad_centers"), (gq, "grad_conics"), (feats, "grad_features"),
                     (gabs, "grad_abs"), (gp, "grad_planes"), (gn, "grad_normals")):
        assert rel_l2(got.cpu().numpy(), g[ref]) <= 1e-3, ref


def test_rade_render_backward_partial_upstreams(golden):
    """Each upstream image alone (the others None, as autograd passes unused
    outputs) against the oracle."""
    g = golden
    W, H = int(g["width"]), int(g["height"])
    st = _golden_state(g)
    bins = dict(ranges=_t(g["ranges"]), point_list=_t(g["ids"]))
    extras = _t(g["extras"]) if g["extras"].shape[1] else None
    feats = np.concatenate([g["colors"], g["extras"]], 1)
    fwd = _forward_from_planar(g)
    names = ("up_features", "up_alpha", "up_depth", "up_median", "up_normals")
    for k, name in enumerate(names):
        ups = [None] * 5
        ups[k] = _t(g[name])
        gc, gq, ga, gb, gp, gn, _ = rrender.backward(
            st, bins, _t(g["colors"]), extras, _t(g["background"]), _t(g["K"]), fwd, tuple(ups),
            W, H)
        ref = O.rade_render_backward(
            W, H, g["ranges"], g["ids"], g["centers"], g["conics"], feats, g["background"],
            g["planes"], g["normals"], g["K"], g["image"], g["auxiliary"], g["contributors"],
            *[g[n] if i == k else None for i, n in enumerate(names)], absgrad=False)
        got_f = ga if gb is None else torch.cat([ga, gb], 1)
        for got, key in ((gc, "centers"), (gq, "conics"), (got_f, "features"), (gp, "planes"),
                         (gn, "normals")):
            if np.abs(ref[key]).max() == 0:
                assert not got.any(), (name, key)
            else:
                assert rel_l2(got.cpu().numpy(), ref[key]) <= 1e-3, (name, key)


def test_rade_projection_backward_matches_autograd_oracle(golden):
    g = golden
    W, H = int(g["width"]), int(g["height"])
    n = len(g["means"])
    rng = np.random.default_rng(21)
    seeds = [rng.standard_normal((n, k)).astype(np.float32) for k in (2, 4, 3, 3)]
    seeds[1] *= 1e-2
    st = _project(g)
    grads = rproj.backward(_t(g["means"]), _t(g["quats"]), _t(g["scales"]), _t(g["opacities"]),
                           _t(g["viewmat"]), _t(g["full"]), _t(g["K"]), _config(g), st,
                           *[_t(s) for s in seeds], (True,) * 6)
    ref = rade_vjp.project_backward(g["means"], g["quats"], g["scales"], g["opacities"],
                                    g["viewmat"], g["full"], g["K"], W, H, g["radii"], *seeds,
                                    kernel_size=float(g["kernel_size"]), planes=g["planes"])
    vis = g["radii"] > 0
    for got, want, name in zip(grads, ref, ("means", "quats", "scales", "opacities", "view",
                                            "proj")):
        got = got.cpu().numpy()
        if name in ("view", "proj"):
            assert rel_l2(got, want) <= 1e-3, name
        else:
            assert not got[~vis].any(), name
            assert rel_l2(got[vis], want[vis]) <= 1e-3, name


def test_rade_rasterize_api_matches_oracle(golden):
    """rade.rasterize with the golden scene's colours as features (extra
    channels get the API's zero background, rade/autograd.py:44-47): the
    images equal the oracle's, and the gradients equal the oracle's render
    backward composed with the projection VJP oracle."""
    g = golden
    W, H = int(g["width"]), int(g["height"])
    C = g["colors"].shape[1]
    E = g["extras"].shape[1]
    means = _t(g["means"]).requires_grad_()
    quats = _t(g["quats"]).requires_grad_()
    scales = _t(g["scales"]).requires_grad_()
    opac = _t(g["opacities"]).requires_grad_()
    colors = _t(g["colors"]).requires_grad_()
    extras = _t(g["extras"]).requires_grad_() if E else None
    res = rade.rasterize(means, quats, scales, opac, _t(g["viewmat"])[None], _t(g["K"])[None],
                         W, H, features=colors, extra_features=extras,
                         backgrounds=_t(g["background"][:C])[None], absgrad=True,
                         kernel_size=float(g["kernel_size"]))
    bg = np.concatenate([g["background"][:C], np.zeros(E, np.float32)])
    feats = np.concatenate([g["colors"], g["extras"]], 1)
    # the oracle projects the quaternions the API normalised (Torch's CUDA
    # F.normalize, inputs.py:252), so that every projected float matches
    qn = torch.nn.functional.normalize(_t(g["quats"]), dim=-1).cpu().numpy()
    geo = O.rade_project(g["means"], qn, g["scales"], g["opacities"], g["viewmat"], g["full"],
                         g["K"], W, H, kernel_size=float(g["kernel_size"]))
    offsets = np.cumsum(geo["tiles"]).astype(np.int32)
    _, ids, ranges = O.bin_and_sort(geo["centers"], geo["radii"], geo["depths"], offsets, W, H)
    image, aux, contrib = O.rade_render(W, H, ranges, ids, geo["centers"], geo["conics"], feats,
                                        bg, geo["planes"], geo["normals"], g["K"])
    img = image.transpose(1, 2, 0)
    np.testing.assert_allclose(res.features[0].detach().cpu().numpy(), img[..., :C], atol=1e-5,
                               rtol=0)
    if E:
        np.testing.assert_allclose(res.extra_features[0].detach().cpu().numpy(),
                                   img[..., C:C + E], atol=1e-5, rtol=0)
    for got, lo in ((res.alpha, 0), (res.depth, 1), (res.median_depth, 2)):
        np.testing.assert_allclose(got[0].detach().cpu().numpy()[..., 0], img[..., C + E + lo],
                                   atol=1e-5, rtol=0)
    np.testing.assert_allclose(res.normals[0].detach().cpu().numpy(), img[..., -3:], atol=1e-5,
                               rtol=0)
    # loss = sum of every output times the golden upstream images
    up_f = _t(g["up_features"])
    loss = (res.features[0] * up_f[..., :C]).sum() + (res.alpha[0] * _t(g["up_alpha"])).sum()
    loss = loss + (res.depth[0] * _t(g["up_depth"])).sum()
    loss = loss + (res.median_depth[0] * _t(g["up_median"])).sum()
    loss = loss + (res.normals[0] * _t(g["up_normals"])).sum()
    if E:
        loss = loss + (res.extra_features[0] * up_f[..., C:]).sum()
    loss.backward()
    want = O.rade_render_backward(W, H, ranges, ids, geo["centers"], geo["conics"], feats, bg,
                                  geo["planes"], geo["normals"], g["K"], image, aux, contrib,
                                  g["up_features"], g["up_alpha"], g["up_depth"],
                                  g["up_median"], g["up_normals"])
    assert rel_l2(colors.grad.cpu().numpy(), want["features"][:, :C]) <= 1e-3
    if E:
        assert rel_l2(extras.grad.cpu().numpy(), want["features"][:, C:]) <= 1e-3
    assert rel_l2(res.means2d.absgrad[0].cpu().numpy(), want["abs"]) <= 1e-3
    assert rel_l2(res.means2d.grad[0].cpu().numpy(), want["centers"]) <= 1e-3
    ref = rade_vjp.project_backward(g["means"], qn, g["scales"], g["opacities"], g["viewmat"],
                                    g["full"], g["K"], W, H, geo["radii"], want["centers"],
                                    want["conics"], want["planes"], want["normals"],
                                    kernel_size=float(g["kernel_size"]), planes=geo["planes"])
    q = qn.astype(np.float64)
    raw = np.linalg.norm(g["quats"].astype(np.float64), axis=1, keepdims=True)
    gq = (ref[1] - q * (q * ref[1]).sum(1, keepdims=True)) / raw  # F.normalize's VJP
    for got, want_g, name in ((means.grad, ref[0], "means"), (quats.grad, gq, "quats"),
                              (scales.grad, ref[2], "scales"), (opac.grad, ref[3], "opacities")):
        assert rel_l2(got.cpu().numpy(), want_g) <= 1e-3, name


def _config4_case(n=40_000, width=400, height=300):
    from dsl_splat_b200.scenes import make_scene

    return make_scene(4, n=n, width=width, height=height, with_grads=False)


def test_rade_config4_shape_against_oracle():
    """A config-4-shaped view (35 blended channels: SH3 colour + 32 extras,
    1200/1600 focal ratio, clustered scene) at reduced size: projection,
    bins and contributors bit-exact, images 1e-5, render gradients 1e-3,
    against the CPU oracle."""
    sc = _config4_case()
    W, H = sc.width, sc.height
    dev = "cuda:0"
    K = sc.Ks[0]
    full, _, campos = stages.cameras_prepare(sc.viewmats.to(dev), sc.Ks.to(dev), W, H, True)
    full_np = full[0].cpu().numpy()
    q = torch.nn.functional.normalize(sc.quats, dim=-1)
    cfg = rproj.ViewConfig(W, H, 0.2, float("inf"), 0.0, "radius", 0.0)
    st = rproj.prepare(sc.means.to(dev), q.to(dev), sc.scales.to(dev), sc.opacities.to(dev),
                       sc.viewmats[0].to(dev), full[0], K.to(dev), cfg)
    ref = O.rade_project(sc.means.numpy(), q.numpy(), sc.scales.numpy(), sc.opacities.numpy(),
                         sc.viewmats[0].numpy(), full_np, K.numpy(), W, H)
    np.testing.assert_array_equal(st.radii.cpu().numpy(), ref["radii"])
    np.testing.assert_array_equal(st.tile_counts.cpu().numpy(), ref["tiles"])
    vis = ref["radii"] > 0
    for name, t in (("centers", st.centers), ("conics", st.conics), ("depths", st.depths),
                    ("planes", st.ray_planes), ("normals", st.normals)):
        np.testing.assert_array_equal(t.cpu().numpy()[vis], ref[name][vis], err_msg=name)
    bins = stages.bin_and_sort(st, W, H)
    offsets = np.cumsum(ref["tiles"]).astype(np.int32)
    _, ids, ranges = O.bin_and_sort(ref["centers"], ref["radii"], ref["depths"], offsets, W, H)
    np.testing.assert_array_equal(bins["ranges"].cpu().numpy(), ranges)
    np.testing.assert_array_equal(bins["point_list"].cpu().numpy(), ids)
    rng = np.random.default_rng(4)
    colors = rng.uniform(0, 1, (sc.means.shape[0], 3)).astype(np.float32)
    extras = sc.extras.numpy()
    bg = rng.uniform(0, 1, 35).astype(np.float32)
    out = rrender.render(st, bins, _t(colors), _t(extras), _t(bg), K.to(dev), W, H)
    feats = np.concatenate([colors, extras], 1)
    image, aux, contrib = O.rade_render(W, H, ranges, ids, ref["centers"], ref["conics"], feats,
                                        bg, ref["planes"], ref["normals"], K.numpy())
    np.testing.assert_array_equal(out.contributors.cpu().numpy(), contrib)
    np.testing.assert_allclose(out.planar().cpu().numpy(), image, atol=1e-5, rtol=1e-6)
    np.testing.assert_allclose(out.auxiliary.cpu().numpy(), aux, atol=1e-5, rtol=1e-6)
    ups = [rng.standard_normal((H, W, k)).astype(np.float32) for k in (35, 1, 1, 1, 3)]
    gc, gq, ga, gb, gp, gn, gabs = rrender.backward(
        st, bins, _t(colors), _t(extras), _t(bg), K.to(dev), out, tuple(_t(u) for u in ups), W,
        H, absgrad=True)
    want = O.rade_render_backward(W, H, ranges, ids, ref["centers"], ref["conics"], feats, bg,
                                  ref["planes"], ref["normals"], K.numpy(), image, aux, contrib,
                                  *ups)
    for got, key in ((gc, "centers"), (gq, "conics"), (torch.cat([ga, gb], 1), "features"),
                     (gabs, "abs"), (gp, "planes"), (gn, "normals")):
        assert rel_l2(got.cpu().numpy(), want[key]) <= 1e-3, key


def test_rade_ops_stages_compose_like_rasterize(golden):
    """rade.ops prepare_gaussians -> bin_and_sort -> rasterize_to_pixels gives
    the oracle's bins and images."""
    from dsl_splat_b200 import PinholeCamera

    g = golden
    W, H = int(g["width"]), int(g["height"])
    cam = PinholeCamera(_t(g["viewmat"]), _t(g["K"]), W, H, 0.2)
    geo = rade.ops.prepare_gaussians(_t(g["means"]), _t(g["quats"]), _t(g["scales"]),
                                     _t(g["opacities"]), cam,
                                     kernel_size=float(g["kernel_size"]))
    tiles = rade.ops.bin_and_sort(geo)
    feats = np.concatenate([g["colors"], g["extras"]], 1)
    px = rade.ops.rasterize_to_pixels(geo, tiles, _t(feats), _t(g["background"]))
    # the oracle on the quaternions prepare_gaussians normalised on the GPU
    qn = torch.nn.functional.normalize(_t(g["quats"]), dim=-1).cpu().numpy()
    ref = O.rade_project(g["means"], qn, g["scales"], g["opacities"], g["viewmat"], g["full"],
                         g["K"], W, H, kernel_size=float(g["kernel_size"]))
    np.testing.assert_array_equal(geo.radii.cpu().numpy(), ref["radii"])
    offsets = np.cumsum(ref["tiles"]).astype(np.int32)
    _, ids, ranges = O.bin_and_sort(ref["centers"], ref["radii"], ref["depths"], offsets, W, H)
    np.testing.assert_array_equal(tiles.gaussian_ids.cpu().numpy(), ids)
    image, _, _ = O.rade_render(W, H, ranges, ids, ref["centers"], ref["conics"], feats,
                                g["background"], ref["planes"], ref["normals"], g["K"])
    img = image.transpose(1, 2, 0)
    np.testing.assert_allclose(px.features.cpu().numpy(), img[..., :-6], atol=1e-5, rtol=0)
    np.testing.assert_allclose(px.depth.cpu().numpy()[..., 0], img[..., -5], atol=1e-5, rtol=0)
    np.testing.assert_allclose(px.normals.cpu().numpy(), img[..., -3:], atol=1e-5, rtol=0)


@pytest.mark.parametrize("name", ["c1_sh3", "dense_sh1"])
def test_rade_fused_sh_matches_composed_sh(name):
    """rade.rasterize(sh_coeffs=...) (projection, SH colours on means - campos
    and metadata in one launch each way) against the composition the
    reference runs: the standalone SH autograd Function on means - campos,
    then rade.rasterize(features=colours).  Images identical to 1e-5 (same
    colour bits); gradients of means, quats, scales, opacities, SH
    coefficients and the view matrix within relative L2 1e-4.  The
    quaternions are not unit length: a third run normalises them with Torch
    first, and the in-kernel normalisation's VJP must give the same quats
    gradient (1e-3)."""
    from dsl_splat_b200.camera_prep import prepare_cameras_with_centers
    from dsl_splat_b200.spherical_harmonics import spherical_harmonics

    g = dict(np.load(os.path.join(ROOT, "tests", "golden", f"rade_{name}.npz")))
    W, H, deg = int(g["width"]), int(g["height"]), int(g["sh_degree"])
    rng = np.random.default_rng(3)
    raw_quats = g["quats"] * rng.uniform(0.5, 2.0, (len(g["quats"]), 1)).astype(np.float32)
    ups = [_t(rng.standard_normal((H, W, k)).astype(np.float32)) for k in (3, 1, 1, 1, 3)]

    def run(mode: str):
        leaves = [_t(g["means"]), _t(raw_quats), _t(g["scales"]), _t(g["opacities"]),
                  _t(g["sh"]), _t(g["viewmat"])[None]]
        for t in leaves:
            t.requires_grad_()
        means, quats, scales, opac, sh, view = leaves
        Ks = _t(g["K"])[None]
        kw = dict(kernel_size=float(g["kernel_size"]), absgrad=True)
        if mode == "fused":
            res = rade.rasterize(means, quats, scales, opac, view, Ks, W, H, sh_coeffs=sh,
                                 sh_degree=deg, **kw)
        else:
            with torch.no_grad():
                radii = rade.rasterize(means, quats, scales, opac, view, Ks, W, H,
                                       features=_t(g["colors"]), **kw).radii[0, :, 0]
            _, campos = prepare_cameras_with_centers(view, Ks, W, H)
            colors = spherical_harmonics(sh, (means - campos[0]).contiguous(), deg,
                                         radii=radii.contiguous())
            q = torch.nn.functional.normalize(quats, dim=-1) if mode == "normalize" else quats
            res = rade.rasterize(means, q, scales, opac, view, Ks, W, H, features=colors, **kw)
        outs = (res.features[0], res.alpha[0], res.depth[0], res.median_depth[0],
                res.normals[0])
        torch.autograd.backward(outs, ups)
        return [o.detach().cpu().numpy() for o in outs], [t.grad.cpu().numpy() for t in leaves]

    fused_out, fused_grads = run("fused")
    ref_out, ref_grads = run("sh")
    for a, b in zip(fused_out, ref_out):
        np.testing.assert_allclose(a, b, atol=1e-5, rtol=0)
    for a, b, what in zip(fused_grads, ref_grads,
                          ("means", "quats", "scales", "opacities", "sh", "viewmat")):
        assert rel_l2(a, b) <= 1e-4, what
    _, torch_grads = run("normalize")
    assert rel_l2(fused_grads[1], torch_grads[1]) <= 1e-3


def test_rade_statistics_add_up_to_alpha(golden):
    """rade.rasterize's contribution statistics (statistics.py:47-73 through
    the rade blend): a weighted sum with pixel weights v adds v * alpha * T
    per blended sample, so its total over Gaussians is sum_p v_p alpha_p (the
    blend weights of a pixel sum to 1 - T_final); a masked count counts the
    blended samples of the masked pixels, at least one per covered pixel."""
    from dsl_splat_b200 import MaskedContributionCount, WeightedContributionSum

    g = golden
    W, H = int(g["width"]), int(g["height"])
    dev = torch.device("cuda", 0)
    half = torch.zeros(H, W, dtype=torch.bool, device=dev)
    half[: H // 2] = True
    ramp = torch.linspace(0.0, 1.0, H * W, device=dev).reshape(H, W)
    res = rade.rasterize(
        _t(g["means"]), _t(g["quats"]), _t(g["scales"]), _t(g["opacities"]),
        _t(g["viewmat"])[None], _t(g["K"])[None], W, H, features=_t(g["colors"]),
        kernel_size=float(g["kernel_size"]),
        statistics=[WeightedContributionSum("ones", torch.ones(H, W, device=dev)),
                    MaskedContributionCount("top", half),
                    WeightedContributionSum("ramp", ramp)])
    alpha = res.alpha[0, ..., 0].double()
    for name, weights in (("ones", torch.ones_like(alpha)), ("ramp", ramp.double())):
        total = res.statistics[name][0].double().sum()
        want = (weights * alpha).sum()
        assert abs(float(total - want)) <= 1e-4 * float(want), name
    counts = res.statistics["top"][0]
    assert counts.dtype == torch.int32 and int(counts.min()) >= 0
    covered = int(((alpha > 0) & half).sum())
    assert int(counts.sum()) >= covered > 0


def test_rade_gsplat_adapter_modes_and_packed_metadata(golden):
    """rade.gsplat.rasterization (rade/gsplat.py:82-191): RGB+ED appends the
    expected depth, D is depth times alpha, and with its default packed=True
    the means2d gradient and absgrad rows are the visible rows of the dense
    API's (same call, packed=False)."""
    from dsl_splat_b200.rade.gsplat import rasterization

    g = golden
    W, H = int(g["width"]), int(g["height"])
    ks = float(g["kernel_size"])

    def call(packed, mode):
        means = _t(g["means"]).requires_grad_()
        args = (means, _t(g["quats"]), _t(g["scales"]), _t(g["opacities"]), _t(g["colors"]),
                _t(g["viewmat"])[None], _t(g["K"])[None], W, H)
        image, alpha, meta = rasterization(*args, near_plane=0.2, eps2d=ks, packed=packed,
                                           render_mode=mode, absgrad=True)
        (image * image).sum().backward()
        return image, alpha, meta, means

    dense_img, dense_alpha, dense_meta, _ = call(False, "RGB+ED")
    packed_img, packed_alpha, packed_meta, _ = call(True, "RGB+ED")
    assert dense_img.shape[-1] == 4
    torch.testing.assert_close(packed_img, dense_img, atol=1e-5, rtol=0)
    torch.testing.assert_close(dense_img[..., 3:], dense_meta["depth"], atol=0, rtol=0)
    d_img, d_alpha, _, _ = call(False, "D")
    torch.testing.assert_close(d_img, dense_meta["depth"] * dense_alpha, atol=1e-5, rtol=1e-6)
    ids = packed_meta["gaussian_ids"]
    vis = (dense_meta["radii"][0] > 0).all(-1)
    assert torch.equal(ids, vis.nonzero()[:, 0])
    for key in ("grad", "absgrad"):
        dense = getattr(dense_meta["means2d"], key)[0]
        packed = getattr(packed_meta["means2d"], key)
        assert rel_l2(packed.cpu().numpy(), dense[ids].cpu().numpy()) <= 1e-5, key
        assert not dense[~vis].any(), key


@pytest.mark.parametrize("case", ["empty", "behind_camera"])
def test_rade_rasterize_empty_and_culled(case):
    """No Gaussians, or only Gaussians behind the camera: the features are the
    background, alpha, both depths and the normals are zero, nothing is
    culled wrongly into view, and the backward runs and gives zero
    gradients (rade/render.py:202-227: uncovered pixels keep zero depth and
    normal)."""
    dev = torch.device("cuda", 0)
    W, H, n = 40, 24, (0 if case == "empty" else 50)
    g = torch.Generator().manual_seed(8)
    means = torch.randn(n, 3, generator=g)
    means[:, 2] = -2.0 - torch.rand(n, generator=g)  # behind an identity camera
    means = means.to(dev).requires_grad_()
    quats = torch.randn(n, 4, generator=g).to(dev).requires_grad_()
    scales = torch.full((n, 3), 0.1).to(dev).requires_grad_()
    opac = torch.full((n,), 0.8).to(dev).requires_grad_()
    colors = torch.rand(n, 3, generator=g).to(dev).requires_grad_()
    K = torch.tensor([[40.0, 0.0, 20.0], [0.0, 40.0, 12.0], [0.0, 0.0, 1.0]], device=dev)
    bg = torch.tensor([0.2, 0.4, 0.6], device=dev)
    res = rade.rasterize(means, quats, scales, opac, torch.eye(4, device=dev)[None], K[None], W,
                         H, features=colors, backgrounds=bg[None], absgrad=True)
    assert torch.equal(res.features[0], bg.expand(H, W, 3))
    for image in (res.alpha, res.depth, res.median_depth, res.normals):
        assert not image.any()
    assert not res.radii.any()
    loss = (res.features.sum() + res.alpha.sum() + res.depth.sum() + res.median_depth.sum()
            + res.normals.sum())
    loss.backward()
    for leaf in (means, quats, scales, opac, colors):
        assert leaf.grad is None or not leaf.grad.any()
