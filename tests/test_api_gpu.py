"""gs3d.rasterize / gsplat.rasterization end to end against the oracle.

The oracle composes the reference's per-view chain (gs3d/api.py:47-265,
gs3d/autograd.py:19-171): camera preparation, projection, masked SH,
binning, blending and their VJPs; per-view gradients are summed as Torch
autograd does for shared parameters.  Quaternion normalisation is a Torch op
in both (inputs.py:252), so its VJP is applied with Torch on the CPU.
Tolerances: images max-abs 1e-5, gradients relative L2 1e-3.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import rel_l2
from dsl_splat_b200 import gs3d
from dsl_splat_b200.gs3d.gsplat import rasterization
from dsl_splat_b200.scenes import make_scene
from oracle import oracle as O

pytestmark = pytest.mark.gpu

IMG_TOL = 1e-5
GRAD_TOL = 1e-3


def _run(scene, *, use_features=False, absgrad=True, background=None, tile_mode="radius"):
    d = torch.device("cuda", 0)
    p = {k: getattr(scene, k).to(d).requires_grad_(True)
         for k in ("means", "quats", "scales", "opacities")}
    viewmats = scene.viewmats.to(d).requires_grad_(True)
    Ks = scene.Ks.to(d)
    kw = {}
    if use_features:
        colors = scene.sh_coeffs[:, 0].to(d).contiguous().requires_grad_(True)
        kw["features"] = colors
    else:
        colors = scene.sh_coeffs.to(d).requires_grad_(True)
        kw["sh_coeffs"] = colors
    if background is not None:
        kw["backgrounds"] = background.to(d)
    res = gs3d.rasterize(p["means"], p["quats"], p["scales"], p["opacities"], viewmats, Ks,
                         scene.width, scene.height, absgrad=absgrad, tile_mode=tile_mode, **kw)
    C = scene.viewmats.shape[0]
    g = torch.Generator().manual_seed(11)
    gF = torch.randn(C, scene.height, scene.width, 3, generator=g)
    gA = torch.randn(C, scene.height, scene.width, 1, generator=g)
    loss = (res.features * gF.to(d)).sum() + (res.alpha * gA.to(d)).sum()
    loss.backward()
    return res, p, viewmats, colors, gF, gA


def _oracle(scene, gF, gA, *, use_features=False, background=None, tile_mode="radius"):
    d = torch.device("cuda", 0)
    qn_gpu = F.normalize(scene.quats.to(d), dim=-1).cpu()
    C = scene.viewmats.shape[0]
    means = scene.means.numpy()
    qn = qn_gpu.numpy()
    acc = None
    images, per_view = [], []
    for c in range(C):
        kw = dict(features=scene.sh_coeffs[:, 0].numpy()) if use_features else dict(
            sh_coeffs=scene.sh_coeffs.numpy(), sh_degree=scene.sh_degree)
        r, bg = O.gs3d_view_forward(means, qn, scene.scales.numpy(), scene.opacities.numpy(),
                                    scene.viewmats[c].numpy(), scene.Ks[c].numpy(), scene.width,
                                    scene.height, background=None if background is None else
                                    background[c].numpy(), tile_mode=tile_mode, **kw)
        up = np.concatenate([gF[c].numpy(), gA[c].numpy()], axis=-1)
        if use_features:
            g = O.gs3d_view_backward(r, bg, means, qn, scene.scales.numpy(),
                                     scene.opacities.numpy(), scene.viewmats[c].numpy(),
                                     scene.Ks[c].numpy(), scene.width, scene.height, up)
        else:
            g = O.gs3d_view_backward(r, bg, means, qn, scene.scales.numpy(),
                                     scene.opacities.numpy(), scene.viewmats[c].numpy(),
                                     scene.Ks[c].numpy(), scene.width, scene.height, up,
                                     sh_coeffs=scene.sh_coeffs.numpy(), sh_degree=scene.sh_degree)
        images.append(r.image)
        per_view.append(g)
        vals = dict(means=g.means, quats_n=g.quats_n, scales=g.scales, opacities=g.opacities,
                    colors=g.sh if not use_features else g.colors)
        acc = vals if acc is None else {k: acc[k] + v for k, v in vals.items()}
    _, vjp = torch.func.vjp(lambda q: F.normalize(q, dim=-1), scene.quats.double())
    acc["quats"] = vjp(torch.from_numpy(np.asarray(acc["quats_n"], np.float64)))[0].numpy()
    return images, per_view, acc


CASES = {
    "c0_sh0": (dict(config=0), False),
    "c0_features": (dict(config=0), True),
    "c1_small_sh3": (dict(config=1, n=20000, width=480, height=270), False),
    "c2_three_views": (dict(config=2, n=30000, width=324, height=210, cameras=3), False),
}


@pytest.mark.parametrize("case", list(CASES))
def test_rasterize_forward_backward(case):
    cfg, use_features = CASES[case]
    scene = make_scene(**cfg)
    bg = None
    if case == "c0_features":
        bg = torch.tensor([[0.2, 0.4, 0.6]])
    res, p, viewmats, colors, gF, gA = _run(scene, use_features=use_features, background=bg)
    images, per_view, acc = _oracle(scene, gF, gA, use_features=use_features, background=bg)
    C = scene.viewmats.shape[0]
    got = torch.cat([res.features, res.alpha], -1).detach().cpu().numpy()
    for c in range(C):
        assert np.abs(np.moveaxis(got[c], -1, 0) - images[c]).max() <= IMG_TOL
    assert rel_l2(p["means"].grad.cpu(), acc["means"]) <= GRAD_TOL
    assert rel_l2(p["quats"].grad.cpu(), acc["quats"]) <= GRAD_TOL
    assert rel_l2(p["scales"].grad.cpu(), acc["scales"]) <= GRAD_TOL
    assert rel_l2(p["opacities"].grad.cpu(), acc["opacities"]) <= GRAD_TOL
    assert rel_l2(colors.grad.cpu(), acc["colors"]) <= GRAD_TOL
    for c in range(C):
        assert rel_l2(viewmats.grad[c].cpu(), per_view[c].viewmat) <= GRAD_TOL
        assert rel_l2(res.means2d.grad[c].cpu(), per_view[c].means2d) <= GRAD_TOL
        assert rel_l2(res.means2d.absgrad[c].cpu(), per_view[c].absgrad) <= GRAD_TOL
    radii = res.radii.cpu().numpy()
    assert radii.shape == (C, scene.means.shape[0], 2)


def test_packed_metadata_and_gsplat_adapter():
    scene = make_scene(0, n=2000)
    d = torch.device("cuda", 0)
    means = scene.means.to(d).requires_grad_(True)
    feats, alpha, meta = rasterization(
        means, scene.quats.to(d), scene.scales.to(d), scene.opacities.to(d),
        scene.sh_coeffs.to(d), scene.viewmats.to(d), scene.Ks.to(d), scene.width, scene.height,
        sh_degree=0, packed=True, absgrad=True, near_plane=0.2)
    dense = gs3d.rasterize(means, scene.quats.to(d), scene.scales.to(d), scene.opacities.to(d),
                           scene.viewmats.to(d), scene.Ks.to(d), scene.width, scene.height,
                           sh_coeffs=scene.sh_coeffs.to(d), packed=False)
    assert torch.equal(feats, dense.features)
    vis = (dense.radii[0] > 0).all(-1)
    assert meta["packed"] is True
    assert len(meta["means2d"]) == int(vis.sum())
    assert torch.equal(meta["gaussian_ids"], vis.nonzero().flatten())
    (feats.sum() + alpha.sum()).backward()
    assert meta["means2d"].grad is not None
    assert meta["means2d"].absgrad.shape == meta["means2d"].shape


def test_statistics_counts_and_sums():
    from dsl_splat_b200 import MaskedContributionCount, WeightedContributionSum
    scene = make_scene(0, n=3000)
    d = torch.device("cuda", 0)
    H, W = scene.height, scene.width
    mask = torch.zeros(H, W, dtype=torch.bool, device=d)
    mask[: H // 2] = True
    weights = torch.rand(H, W, device=d)
    res = gs3d.rasterize(scene.means.to(d), scene.quats.to(d), scene.scales.to(d),
                         scene.opacities.to(d), scene.viewmats.to(d), scene.Ks.to(d), W, H,
                         sh_coeffs=scene.sh_coeffs.to(d),
                         statistics=(MaskedContributionCount("hits", mask),
                                     WeightedContributionSum("score", weights)))
    hits = res.statistics["hits"]
    score = res.statistics["score"]
    assert hits.shape == (1, 3000) and score.shape == (1, 3000)
    # full-image weights of one reproduce sum over pixels of alpha*T per Gaussian
    ones = torch.ones(H, W, device=d)
    res2 = gs3d.rasterize(scene.means.to(d), scene.quats.to(d), scene.scales.to(d),
                          scene.opacities.to(d), scene.viewmats.to(d), scene.Ks.to(d), W, H,
                          sh_coeffs=scene.sh_coeffs.to(d),
                          statistics=(WeightedContributionSum("w", ones),))
    total = float(res2.statistics["w"].sum())
    alpha_sum = float(res2.alpha.sum())
    assert abs(total - alpha_sum) <= 1e-3 * max(1.0, alpha_sum)
    assert int(hits.sum()) > 0 and float(score.sum()) > 0


def test_error_paths():
    scene = make_scene(0, n=100)
    d = torch.device("cuda", 0)
    args = [scene.means.to(d), scene.quats.to(d), scene.scales.to(d), scene.opacities.to(d),
            scene.viewmats.to(d)]
    bad_k = scene.Ks.clone()
    bad_k[0, 0, 0] = -1.0
    with pytest.raises(ValueError, match="positive fx/fy"):
        gs3d.rasterize(*args, bad_k.to(d), scene.width, scene.height, sh_coeffs=scene.sh_coeffs.to(d))
    skew = scene.Ks.clone()
    skew[0, 0, 1] = 0.5
    with pytest.raises(NotImplementedError, match="zero-skew"):
        gs3d.rasterize(*args, skew.to(d), scene.width, scene.height, sh_coeffs=scene.sh_coeffs.to(d))
    sh3 = torch.zeros(100, 16, 3, device=d)
    singular = torch.zeros(1, 4, 4, device=d)
    with pytest.raises(torch.linalg.LinAlgError):
        gs3d.rasterize(args[0], args[1], args[2], args[3], singular, scene.Ks.to(d), scene.width,
                       scene.height, sh_coeffs=sh3)


@pytest.mark.parametrize("tile_mode", ["snugbox", "accutile"])
def test_rasterize_tile_modes(tile_mode):
    """gs3d.rasterize(tile_mode=...) end to end: images, gradients and the
    tiles_per_gauss metadata of the mode against the oracle."""
    scene = make_scene(config=1, n=20000, width=480, height=270)
    res, p, viewmats, colors, gF, gA = _run(scene, tile_mode=tile_mode)
    images, per_view, acc = _oracle(scene, gF, gA, tile_mode=tile_mode)
    got = torch.cat([res.features, res.alpha], -1).detach().cpu().numpy()
    assert np.abs(np.moveaxis(got[0], -1, 0) - images[0]).max() <= IMG_TOL
    for name in ("means", "quats", "scales", "opacities"):
        assert rel_l2(p[name].grad.cpu(), acc[name]) <= GRAD_TOL, name
    assert rel_l2(colors.grad.cpu(), acc["colors"]) <= GRAD_TOL
    assert res.meta["tile_mode"] == tile_mode
    qn = F.normalize(scene.quats.to("cuda:0"), dim=-1).cpu().numpy()
    full, _, _, _ = O.cameras_prepare(scene.viewmats[:1].numpy(), scene.Ks[:1].numpy(),
                                      scene.width, scene.height, False)
    ref = O.project_forward(scene.means.numpy(), qn, scene.scales.numpy(),
                            scene.opacities.numpy(), scene.viewmats[0].numpy(), full[0],
                            scene.Ks[0].numpy(), scene.width, scene.height, tile_mode=tile_mode)
    np.testing.assert_array_equal(res.meta["tiles_per_gauss"][0].cpu().numpy(), ref.tiles)


def test_single_host_synchronisation_per_call():
    """One host wait per rasterize call (pair counts, camera status and, when
    packed, the visible counts together), as the reference's single .item()
    (primitives/tiling.py:64); packed metadata adds none.  The wait is on an
    event recorded right after the counts' copy to pinned memory, not on the
    stream, so work queued after the copy (the chunked emits) keeps running:
    no stream synchronisation at all, and exactly one event wait."""
    import warnings
    scene = make_scene(config=2, n=30000, width=324, height=210, cameras=3)
    d = torch.device("cuda", 0)
    args = [getattr(scene, k).to(d) for k in ("means", "quats", "scales", "opacities")]
    vm, Ks, sh = scene.viewmats.to(d), scene.Ks.to(d), scene.sh_coeffs.to(d)
    waits = []
    original = torch.cuda.Event.synchronize

    def counted(self):
        waits.append(self)
        return original(self)

    for packed in (False, True):
        gs3d.rasterize(*args, vm, Ks, scene.width, scene.height, sh_coeffs=sh, packed=packed,
                       absgrad=True)  # warm-up (allocator, first-use setup)
        torch.cuda.synchronize()
        waits.clear()
        torch.cuda.set_sync_debug_mode("warn")
        torch.cuda.Event.synchronize = counted
        try:
            with warnings.catch_warnings(record=True) as caught:
                warnings.simplefilter("always")
                res = gs3d.rasterize(*args, vm, Ks, scene.width, scene.height, sh_coeffs=sh,
                                     packed=packed, absgrad=True)
        finally:
            torch.cuda.set_sync_debug_mode(0)
            torch.cuda.Event.synchronize = original
        syncs = [w for w in caught if "synchroniz" in str(w.message)]
        assert not syncs, [str(w.message)[:120] for w in syncs]
        assert len(waits) == 1
        if packed:
            dense = gs3d.rasterize(*args, vm, Ks, scene.width, scene.height, sh_coeffs=sh,
                                   absgrad=True)
            mask = (dense.radii > 0).all(-1)
            assert torch.equal(res.meta["radii"], dense.radii[mask])
            assert torch.equal(res.meta["means2d"].detach(), dense.means2d.detach()[mask])


def test_means2d_gradient_targets_multi_view():
    """means2d.grad (written by the render backward straight into the leaf's
    gradient, dense or packed) equals autograd's per-view routing: the packed
    leaf's rows are the dense gradient at (camera_ids, gaussian_ids), and a
    second backward through the same graph accumulates."""
    scene = make_scene(2, n=20000, width=324, height=210, cameras=3)
    d = torch.device("cuda", 0)
    args = [t.to(d) for t in (scene.means, scene.quats, scene.scales, scene.opacities)]
    args[0].requires_grad_(True)
    views, Ks = scene.viewmats.to(d), scene.Ks.to(d)
    sh = scene.sh_coeffs.to(d)
    up = scene.grad_image.to(d)
    dense = gs3d.rasterize(*args, views, Ks, scene.width, scene.height, sh_coeffs=sh,
                           absgrad=True)
    dense.features.backward(up, retain_graph=True)
    g_dense = dense.means2d.grad.clone()
    assert g_dense.shape == (3, 20000, 2) and g_dense.abs().sum() > 0
    packed = gs3d.rasterize(*args, views, Ks, scene.width, scene.height, sh_coeffs=sh,
                            absgrad=True, packed=True)
    packed.features.backward(up)
    meta = packed.meta
    # two backward passes differ only in the order of their atomic additions
    want = g_dense[meta["camera_ids"], meta["gaussian_ids"]]
    assert rel_l2(meta["means2d"].grad.cpu(), want.cpu()) <= 1e-5
    assert rel_l2(meta["means2d"].absgrad.cpu(),
                  dense.means2d.absgrad[meta["camera_ids"], meta["gaussian_ids"]].cpu()) <= 1e-5
    dense.features.backward(up)
    assert rel_l2(dense.means2d.grad.cpu(), 2 * g_dense.cpu()) <= 1e-5


@pytest.mark.parametrize("tile_mode,packed", [("radius", False), ("snugbox", True),
                                              ("accutile", False)])
def test_multi_view_call_matches_per_view_calls(tile_mode, packed):
    """A multi-camera rasterize call (one projection launch each way for all
    cameras) renders the same images, radii and means2d, bit for bit, as one
    single-camera call per view, and its Gaussian gradients equal the sum of
    theirs (relative L2 1e-5: summation order only)."""
    scene = make_scene(2, n=20000, width=324, height=210, cameras=3)
    d = torch.device("cuda", 0)

    def leaves():
        return [t.to(d).requires_grad_(True) for t in
                (scene.means, scene.quats, scene.scales, scene.opacities, scene.sh_coeffs)]

    vm, Ks = scene.viewmats.to(d), scene.Ks.to(d)
    up = scene.grad_image.to(d)
    multi = leaves()
    res = gs3d.rasterize(*multi[:4], vm, Ks, scene.width, scene.height, sh_coeffs=multi[4],
                         tile_mode=tile_mode, packed=packed, absgrad=True)
    res.features.backward(up)
    single = leaves()
    for c in range(3):
        one = gs3d.rasterize(*single[:4], vm[c:c + 1], Ks[c:c + 1], scene.width, scene.height,
                             sh_coeffs=single[4], tile_mode=tile_mode, packed=packed,
                             absgrad=True)
        assert torch.equal(one.features[0], res.features[c])
        assert torch.equal(one.alpha[0], res.alpha[c])
        if not packed:
            assert torch.equal(one.radii[0], res.radii[c])
            assert torch.equal(one.means2d[0].detach(), res.means2d[c].detach())
        one.features.backward(up[c:c + 1])
    for a, b in zip(multi, single):
        assert rel_l2(a.grad.cpu(), b.grad.cpu()) <= 1e-5
