"""Parity at the BASELINE configurations' own sizes (not downscaled).

The CUDA path against the CPU oracle on the benchmark scenes themselves:

* config 1 -- 1M Gaussians, SH3, 1920x1080, absgrad (the headline metric's
  workload): every stage, then gs3d.rasterize end to end;
* config 2 -- 3M Gaussians, SH3, 1296x840: one full view stage by stage,
  then the sum over three of its eight orbit views through gs3d.rasterize;
* config 3 -- AAA-Gaussians, 2M Gaussians, SH3, 1920x1080, absgrad:
  aaa.rasterize forward and backward against the oracle's composition
  (SH colours, preprocessing, remainder cull, emission and sort, HIER blend,
  replay, both adjoints, SH backward);
* config 4 -- RaDe-GS, 1M Gaussians, SH3 + 32 extra channels, 1600x1200:
  projection, bins, blend and blend backward, and the projection VJP on a
  fixed band of Gaussian rows against the float64 autograd oracle.

Tolerances (as every parity test here): radii, tile counts, point_list,
ranges, contributor counts and final transmittance bit-exact; projected
floats bit-exact; images max-abs 1e-5; gradients relative L2 1e-3.
"""

import numpy as np
import pytest
import torch

from conftest import rel_l2
from dsl_splat_b200 import stages
from dsl_splat_b200.rade import projection as rproj
from dsl_splat_b200.rade import render as rrender
from dsl_splat_b200.scenes import make_scene
from oracle import oracle as O
from oracle import rade_vjp
from test_api_gpu import _oracle as api_oracle
from test_api_gpu import _run as api_run
from test_parity_gpu import Prepared, _oracle_view

pytestmark = pytest.mark.gpu

IMG_TOL = 1e-5
GRAD_TOL = 1e-3


def _dev():
    return torch.device("cuda", 0)


def _stages_against_oracle(scene, view=0):
    """Projection + SH, binning, blend forward and backward of one view."""
    p = Prepared(scene, view)
    out = p.project()
    r, bg = _oracle_view(p)
    radii = out.state.radii.cpu().numpy()
    np.testing.assert_array_equal(radii, r.proj.radii)
    np.testing.assert_array_equal(out.state.tile_counts.cpu().numpy(), r.proj.tiles)
    vis = radii > 0
    for got, want in ((out.state.centers, r.proj.centers), (out.state.conics, r.proj.conics),
                      (out.state.depths, r.proj.depths)):
        np.testing.assert_array_equal(got.cpu().numpy()[vis], want[vis])
    np.testing.assert_array_equal(out.colors.cpu().numpy(), r.features[:, :3])
    bins = stages.bin_and_sort(out.state, p.W, p.H)
    ids = bins["point_list"].cpu().numpy()
    assert len(ids) == int(r.proj.tiles[vis].sum()) == len(r.ids)
    np.testing.assert_array_equal(bins["ranges"].cpu().numpy(), r.ranges)
    np.testing.assert_array_equal(ids, r.ids)
    bg_t = torch.from_numpy(bg).to(_dev())
    px = stages.render(out.state, bins, out.colors, None, True, bg_t, p.W, p.H)
    np.testing.assert_array_equal(px.contributors.cpu().numpy(), r.contributors)
    np.testing.assert_array_equal(px.transmittance.cpu().numpy(), r.final_t)
    img = np.moveaxis(px.features.cpu().numpy(), -1, 0)
    assert np.abs(img - r.image).max() <= IMG_TOL
    up = np.random.default_rng(17).standard_normal((p.H, p.W, 4)).astype(np.float32)
    gc, gq, ga, _, gabs = stages.render_backward(
        out.state, bins, out.colors, None, True, bg_t, px.transmittance, px.contributors,
        torch.from_numpy(up).to(_dev()), p.W, p.H, absgrad=True, constant_tail=1)
    rc, rq, rf, rabs = O.render_backward(p.W, p.H, r.ranges, r.ids, r.proj.centers,
                                         r.proj.conics, r.features, bg, r.final_t,
                                         r.contributors, np.moveaxis(up, -1, 0).copy(),
                                         absgrad=True, constant_tail=1)
    assert rel_l2(gc.cpu().numpy(), rc) <= GRAD_TOL
    assert rel_l2(gq.cpu().numpy(), rq) <= GRAD_TOL
    assert rel_l2(ga.cpu().numpy(), rf[:, :3]) <= GRAD_TOL
    assert rel_l2(gabs.cpu().numpy(), rabs) <= GRAD_TOL
    return len(ids)


def _api_against_oracle(scene):
    """gs3d.rasterize forward + backward against the oracle's per-view chain
    (gradients summed over the views as autograd does)."""
    res, p, viewmats, colors, gF, gA = api_run(scene)
    images, per_view, acc = api_oracle(scene, gF, gA)
    got = torch.cat([res.features, res.alpha], -1).detach().cpu().numpy()
    for c in range(scene.viewmats.shape[0]):
        assert np.abs(np.moveaxis(got[c], -1, 0) - images[c]).max() <= IMG_TOL
        assert rel_l2(viewmats.grad[c].cpu(), per_view[c].viewmat) <= GRAD_TOL
        assert rel_l2(res.means2d.grad[c].cpu(), per_view[c].means2d) <= GRAD_TOL
        assert rel_l2(res.means2d.absgrad[c].cpu(), per_view[c].absgrad) <= GRAD_TOL
    for name in ("means", "quats", "scales", "opacities"):
        assert rel_l2(p[name].grad.cpu(), acc[name]) <= GRAD_TOL, name
    assert rel_l2(colors.grad.cpu(), acc["colors"]) <= GRAD_TOL


def test_config1_full_stages():
    m = _stages_against_oracle(make_scene(1))
    assert m > 5_000_000  # the headline scene's pair count (9.2M)


def test_config1_full_rasterize():
    _api_against_oracle(make_scene(1))


def test_config2_full_view_stages():
    _stages_against_oracle(make_scene(2), view=0)


def test_config2_three_view_sum():
    scene = make_scene(2)
    keep = [0, 3, 5]  # views on three sides of the orbit
    for name in ("viewmats", "Ks"):
        setattr(scene, name, getattr(scene, name)[keep].contiguous())
    _api_against_oracle(scene)


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(_dev())


def test_config4_full_view():
    sc = make_scene(4, with_grads=False)
    W, H = sc.width, sc.height
    dev = _dev()
    K = sc.Ks[0]
    full, _, _ = stages.cameras_prepare(sc.viewmats.to(dev), sc.Ks.to(dev), W, H, True)
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
    bg = np.zeros(35, np.float32)
    out = rrender.render(st, bins, _t(colors), _t(extras), _t(bg), K.to(dev), W, H)
    feats = np.concatenate([colors, extras], 1)
    image, aux, contrib = O.rade_render(W, H, ranges, ids, ref["centers"], ref["conics"], feats,
                                        bg, ref["planes"], ref["normals"], K.numpy())
    np.testing.assert_array_equal(out.contributors.cpu().numpy(), contrib)
    np.testing.assert_allclose(out.planar().cpu().numpy(), image, atol=IMG_TOL, rtol=0)
    np.testing.assert_allclose(out.auxiliary.cpu().numpy(), aux, atol=IMG_TOL, rtol=0)
    ups = [rng.standard_normal((H, W, k)).astype(np.float32) for k in (35, 1, 1, 1, 3)]
    ups[0] *= 1e-3
    gc, gq, ga, gb, gp, gn, gabs = rrender.backward(
        st, bins, _t(colors), _t(extras), _t(bg), K.to(dev), out, tuple(_t(u) for u in ups), W,
        H, absgrad=True)
    want = O.rade_render_backward(W, H, ranges, ids, ref["centers"], ref["conics"], feats, bg,
                                  ref["planes"], ref["normals"], K.numpy(), image, aux, contrib,
                                  *ups)
    for got, key in ((gc, "centers"), (gq, "conics"), (torch.cat([ga, gb], 1), "features"),
                     (gabs, "abs"), (gp, "planes"), (gn, "normals")):
        assert rel_l2(got.cpu().numpy(), want[key]) <= GRAD_TOL, key
    # projection VJP of the full scene on the GPU, checked on a fixed band of
    # 50k Gaussian rows against float64 autograd (all 1M rows take minutes)
    seeds = [want["centers"], want["conics"], want["planes"], want["normals"]]
    grads = rproj.backward(sc.means.to(dev), q.to(dev), sc.scales.to(dev), sc.opacities.to(dev),
                           sc.viewmats[0].to(dev), full[0], K.to(dev), cfg, st,
                           *[_t(s.astype(np.float32)) for s in seeds], (True,) * 4 + (False,) * 2)
    band = slice(200_000, 250_000)
    ref_g = rade_vjp.project_backward(
        sc.means.numpy()[band], q.numpy()[band], sc.scales.numpy()[band],
        sc.opacities.numpy()[band], sc.viewmats[0].numpy(), full_np, K.numpy(), W, H,
        ref["radii"][band], *[np.ascontiguousarray(s[band]) for s in seeds],
        planes=ref["planes"][band])
    bvis = ref["radii"][band] > 0
    assert bvis.sum() > 10_000
    for got, want_g, name in zip(grads[:4], ref_g[:4], ("means", "quats", "scales", "opacities")):
        g_band = got.cpu().numpy()[band]
        assert rel_l2(g_band[bvis], np.asarray(want_g)[bvis]) <= GRAD_TOL, name


def test_config3_full_aaa():
    import torch.nn.functional as F

    from dsl_splat_b200 import aaa
    dev = _dev()
    sc = make_scene(3)
    W, H = sc.width, sc.height
    leaves = {k: getattr(sc, k).to(dev).requires_grad_(True)
              for k in ("means", "quats", "scales", "opacities", "sh_coeffs")}
    res = aaa.rasterize(leaves["means"], leaves["quats"], leaves["scales"], leaves["opacities"],
                        sc.viewmats.to(dev), sc.Ks.to(dev), W, H,
                        sh_coeffs=leaves["sh_coeffs"], absgrad=True)
    torch.autograd.backward([res.features, res.alpha],
                            [sc.grad_image.to(dev), sc.grad_alpha.to(dev)])
    # the oracle's composition of the same view
    view = aaa.cameras.prepare_cameras(sc.viewmats[None].to(dev), sc.Ks[None].to(dev), W, H,
                                       0.01, 1e10).view(0, 0)
    vargs = (view.viewmatrix.cpu().numpy(), view.projmatrix.cpu().numpy(),
             view.campos.cpu().numpy())
    tanfov = (view.tanfovx, view.tanfovy)
    means, scales, opac = sc.means.numpy(), sc.scales.numpy(), sc.opacities.numpy()
    qn = F.normalize(sc.quats.to(dev), dim=-1).cpu().numpy()  # CUDA F.normalize bits
    pre = O.aaa_preprocess(means, qn, scales, opac, *vargs, W, H, tanfov, view.principal)
    final = O.aaa_cull_remainder(pre, W, H)
    radii = final["radii"]
    np.testing.assert_array_equal((res.radii[0] > 0).any(-1).cpu().numpy(), radii > 0)
    np.testing.assert_array_equal(res.meta["tiles_per_gauss"][0].cpu().numpy(), final["tiles"])
    dirs = means - vargs[2]
    colors, active = O.sh_forward(sc.sh_coeffs.numpy(), dirs, 3)  # aaa/api.py: before culling
    feats = np.concatenate([colors, np.ones((len(means), 1), np.float32)], 1)
    _, keys, values = O.aaa_duplicate(pre, radii, final["tiles"], W, H)
    T = ((W + 15) // 16) * ((H + 15) // 16)
    _, ids, ranges = O.aaa_sort(keys, values, T)
    bg = np.zeros(4, np.float32)
    image, final_t, _ = O.aaa_render(W, H, ranges, ids, pre["transforms"], pre["opacity"],
                                     feats, bg)
    got = torch.cat([res.features, res.alpha], -1)[0].detach().cpu().numpy()
    np.testing.assert_array_equal(np.moveaxis(got, -1, 0), image)
    up = np.concatenate([sc.grad_image[0].numpy(), sc.grad_alpha[0].numpy()], -1)
    g = O.aaa_render_backward(W, H, ranges, ids, pre["transforms"], pre["opacity"], feats, bg,
                              image, final_t, np.moveaxis(up, -1, 0).copy(), screen=True,
                              absgrad=True)
    assert rel_l2(res.means2d.grad[0].cpu(), g["screen"]) <= GRAD_TOL
    assert rel_l2(res.means2d.absgrad[0].cpu(), g["screen_abs"]) <= GRAD_TOL
    up_t, up_o = g["transforms"].astype(np.float32), g["opacity"].astype(np.float32)
    adj = O.aaa_preprocess_backward(means, qn, scales, opac, radii, *vargs, W, H,
                                    np.float32(W / (2.0 * tanfov[0])), up_t, up_o)
    g_sh, g_dirs = O.sh_backward(sc.sh_coeffs.numpy(), dirs, 3, None, active,
                                 g["colors"][:, :3].astype(np.float32))
    assert rel_l2(leaves["sh_coeffs"].grad.cpu(), g_sh) <= GRAD_TOL
    assert rel_l2(leaves["means"].grad.cpu(), adj["means"] + g_dirs) <= GRAD_TOL
    assert rel_l2(leaves["scales"].grad.cpu(), adj["scales"]) <= GRAD_TOL
    assert rel_l2(leaves["opacities"].grad.cpu(), adj["opacity"]) <= GRAD_TOL
    _, vjp = torch.func.vjp(lambda x: F.normalize(x, dim=-1), sc.quats.double())
    gq = vjp(torch.from_numpy(adj["quats"].astype(np.float64)))[0].numpy()
    assert rel_l2(leaves["quats"].grad.cpu(), gq) <= GRAD_TOL
