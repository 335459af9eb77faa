"""The public gs3d stage API (gs3d/ops.py:215-327) on the GPU.

prepare_gaussians -> bin_and_sort -> rasterize_to_pixels with a background
and two statistics requests, forward and backward, against the CPU oracle
(radii, ids and ranges bit-exact, images max-abs 1e-5, gradients relative L2
1e-3) and against gs3d.rasterize on the same inputs (the same kernels: equal
images and statistics, gradients equal up to float32 atomic order).
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import rel_l2
from dsl_splat_b200 import MaskedContributionCount, PinholeCamera, WeightedContributionSum, gs3d
from dsl_splat_b200.scenes import make_scene
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _leaves(scene, d):
    return {k: getattr(scene, k).to(d).requires_grad_(True)
            for k in ("means", "quats", "scales", "opacities")}


def test_gs3d_ops_chain_matches_oracle_and_rasterize():
    d = torch.device("cuda", 0)
    scene = make_scene(1, n=20000, width=480, height=270)
    W, H = scene.width, scene.height
    g = torch.Generator().manual_seed(3)
    feats_np = torch.rand(scene.means.shape[0], 3, generator=g).numpy()
    bg_np = np.array([0.1, 0.5, 0.9], np.float32)
    mask = torch.rand(H, W, generator=g) > 0.5
    weights = torch.rand(H, W, generator=g)
    requests = [MaskedContributionCount("half", mask.to(d)),
                WeightedContributionSum("weighted", weights.to(d))]
    gF = torch.randn(H, W, 3, generator=g).to(d)
    gA = torch.randn(H, W, 1, generator=g).to(d)

    # the stage chain
    p = _leaves(scene, d)
    feats = torch.from_numpy(feats_np).to(d).requires_grad_(True)
    cam = PinholeCamera(scene.viewmats[0].to(d), scene.Ks[0].to(d), W, H, 0.2)
    geo = gs3d.ops.prepare_gaussians(p["means"], p["quats"], p["scales"], p["opacities"], cam)
    tiles = gs3d.ops.bin_and_sort(geo)
    px = gs3d.ops.rasterize_to_pixels(geo, tiles, feats, torch.from_numpy(bg_np).to(d),
                                      statistics=requests)
    ((px.features * gF).sum() + (px.alpha * gA).sum()).backward()

    # the same inputs through gs3d.rasterize
    q = _leaves(scene, d)
    feats2 = torch.from_numpy(feats_np).to(d).requires_grad_(True)
    res = gs3d.rasterize(q["means"], q["quats"], q["scales"], q["opacities"],
                         scene.viewmats.to(d), scene.Ks.to(d), W, H, features=feats2,
                         backgrounds=torch.from_numpy(bg_np).to(d)[None], statistics=requests)
    ((res.features[0] * gF).sum() + (res.alpha[0] * gA).sum()).backward()
    assert torch.equal(px.features, res.features[0])
    assert torch.equal(px.alpha, res.alpha[0])
    # counts are integers (exact); weighted sums are float32 atomics in
    # arbitrary order
    assert torch.equal(px.statistics["half"], res.statistics["half"][0])
    assert rel_l2(px.statistics["weighted"].cpu(), res.statistics["weighted"][0].cpu()) <= 1e-5
    assert int(px.statistics["half"].sum()) > 0
    for name in p:
        assert rel_l2(p[name].grad.cpu(), q[name].grad.cpu()) <= 1e-4, name
    assert rel_l2(feats.grad.cpu(), feats2.grad.cpu()) <= 1e-4

    # the oracle on the quaternions prepare_gaussians normalised on the GPU
    qn = F.normalize(scene.quats.to(d), dim=-1).cpu()
    r, bg = O.gs3d_view_forward(scene.means.numpy(), qn.numpy(), scene.scales.numpy(),
                                scene.opacities.numpy(), scene.viewmats[0].numpy(),
                                scene.Ks[0].numpy(), W, H, features=feats_np, background=bg_np)
    np.testing.assert_array_equal(geo.radii.cpu().numpy(), r.proj.radii)
    np.testing.assert_array_equal(tiles.gaussian_ids.cpu().numpy(), r.ids)
    np.testing.assert_array_equal(tiles.ranges.cpu().numpy(), r.ranges)
    img = np.concatenate([px.features.detach().cpu().numpy(), px.alpha.detach().cpu().numpy()],
                         -1)
    assert np.abs(np.moveaxis(img, -1, 0) - r.image).max() <= 1e-5
    up = np.concatenate([gF.cpu().numpy(), gA.cpu().numpy()], -1)
    want = O.gs3d_view_backward(r, bg, scene.means.numpy(), qn.numpy(), scene.scales.numpy(),
                                scene.opacities.numpy(), scene.viewmats[0].numpy(),
                                scene.Ks[0].numpy(), W, H, up)
    _, vjp = torch.func.vjp(lambda x: F.normalize(x, dim=-1), scene.quats.double())
    gq = vjp(torch.from_numpy(np.asarray(want.quats_n, np.float64)))[0].numpy()
    assert rel_l2(p["means"].grad.cpu(), want.means) <= 1e-3
    assert rel_l2(p["quats"].grad.cpu(), gq) <= 1e-3
    assert rel_l2(p["scales"].grad.cpu(), want.scales) <= 1e-3
    assert rel_l2(p["opacities"].grad.cpu(), want.opacities) <= 1e-3
    assert rel_l2(feats.grad.cpu(), want.colors) <= 1e-3
