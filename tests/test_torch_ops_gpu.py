"""torch.ops.splat200.* on the GPU: the same results as the stage wrappers,
autograd through the operators equal to gs3d.rasterize's gradients, and a
torch.compile trace of the forward chain."""

import pytest
import torch
import torch.nn.functional as F

from conftest import rel_l2
import dsl_splat_b200  # noqa: F401
from dsl_splat_b200 import gs3d, stages
from dsl_splat_b200.scenes import make_scene

pytestmark = pytest.mark.gpu


def _inputs():
    d = torch.device("cuda", 0)
    s = make_scene(1, n=20000, width=480, height=270)
    view, K = s.viewmats[0].to(d).contiguous(), s.Ks[0].to(d).contiguous()
    full, _, campos = torch.ops.splat200.cameras_prepare(view[None], K[None], s.width, s.height,
                                                         True)
    return s, d, view, K, full[0], campos[0]


def _chain(s, d, view, K, full, campos, means, quats_n, scales, opac, sh, tile_mode="radius"):
    ctr, con, radii, tiles, depths = torch.ops.splat200.project(
        means, quats_n, scales, opac, view, full, K, s.width, s.height, 0.2, float("inf"), 0.0,
        tile_mode)
    ranges, ids = torch.ops.splat200.bin_and_sort(ctr, con, radii, tiles, depths, s.width,
                                                  s.height, tile_mode)
    colors, _ = torch.ops.splat200.sh_forward(sh, means - campos, s.sh_degree, radii)
    bg = torch.zeros(4, device=d)
    image, alpha, final_t, contrib = torch.ops.splat200.render(ctr, con, ranges, ids, colors, bg,
                                                               s.width, s.height)
    return image, alpha, final_t, contrib, ranges, ids


@pytest.mark.parametrize("tile_mode", ["radius", "accutile"])
def test_ops_match_stages(tile_mode):
    s, d, view, K, full, campos = _inputs()
    means, q = s.means.to(d), F.normalize(s.quats.to(d), dim=-1)
    scales, opac, sh = s.scales.to(d), s.opacities.to(d), s.sh_coeffs.to(d)
    image, alpha, final_t, contrib, ranges, ids = _chain(s, d, view, K, full, campos, means, q,
                                                         scales, opac, sh, tile_mode)
    st = stages.project(means, q, scales, opac, view, full, K, s.width, s.height, 0.2,
                        float("inf"), 0.0, tile_mode)
    bins = stages.bin_and_sort(st, s.width, s.height, tile_mode=tile_mode)
    assert torch.equal(ranges, bins["ranges"]) and torch.equal(ids, bins["point_list"])
    colors, _ = stages.sh_forward(sh, means - campos, s.sh_degree, st.radii, True)
    px = stages.render(st, bins, colors, None, True, torch.zeros(4, device=d), s.width, s.height,
                       separate_alpha=True)
    assert torch.equal(image, px.features) and torch.equal(alpha, px.alpha)
    assert torch.equal(final_t, px.transmittance) and torch.equal(contrib, px.contributors)


def test_ops_autograd_matches_rasterize():
    s, d, view, K, full, campos = _inputs()
    leaves = {k: getattr(s, k).to(d).requires_grad_(True)
              for k in ("means", "quats", "scales", "opacities")}
    sh = s.sh_coeffs.to(d).requires_grad_(True)
    g = torch.Generator().manual_seed(5)
    gF = torch.randn(s.height, s.width, 3, generator=g).to(d)
    gA = torch.randn(s.height, s.width, 1, generator=g).to(d)
    image, alpha, *_ = _chain(s, d, view, K, full, campos, leaves["means"],
                              F.normalize(leaves["quats"], dim=-1), leaves["scales"],
                              leaves["opacities"], sh)
    ((image * gF).sum() + (alpha * gA).sum()).backward()
    ref = {k: getattr(s, k).to(d).requires_grad_(True)
           for k in ("means", "quats", "scales", "opacities")}
    ref_sh = s.sh_coeffs.to(d).requires_grad_(True)
    res = gs3d.rasterize(ref["means"], ref["quats"], ref["scales"], ref["opacities"],
                         view[None], K[None], s.width, s.height, sh_coeffs=ref_sh,
                         sh_degree=s.sh_degree)
    assert torch.equal(res.features[0], image) and torch.equal(res.alpha[0], alpha)
    ((res.features[0] * gF).sum() + (res.alpha[0] * gA).sum()).backward()
    for k in leaves:
        assert rel_l2(leaves[k].grad.cpu(), ref[k].grad.cpu()) <= 1e-4, k
    assert rel_l2(sh.grad.cpu(), ref_sh.grad.cpu()) <= 1e-4


def test_ops_trace_with_torch_compile():
    s, d, view, K, full, campos = _inputs()
    means, q = s.means.to(d), F.normalize(s.quats.to(d), dim=-1)
    scales, opac, sh = s.scales.to(d), s.opacities.to(d), s.sh_coeffs.to(d)

    def forward(means, q, scales, opac, sh):
        image, alpha, *_ = _chain(s, d, view, K, full, campos, means, q, scales, opac, sh)
        return image, alpha

    eager = forward(means, q, scales, opac, sh)
    torch._dynamo.reset()
    compiled = torch.compile(forward, fullgraph=True, backend="eager")(means, q, scales, opac,
                                                                        sh)
    assert torch.equal(eager[0], compiled[0]) and torch.equal(eager[1], compiled[1])


def test_project_views_op_and_autograd():
    """torch.ops.splat200.project_views returns the stage's stacked outputs,
    and its autograd formula calls project_views_backward with the upstream
    gradients of the stacked centres, conics and colours."""
    from dsl_splat_b200.scenes import make_scene
    d = torch.device("cuda", 0)
    s = make_scene(2, n=5000, width=200, height=130, cameras=3)
    vm, Ks = s.viewmats.to(d), s.Ks.to(d)
    full, _, campos = stages.cameras_prepare(vm, Ks, s.width, s.height, True)
    leaves = [t.to(d).requires_grad_(True) for t in (s.means, s.quats, s.scales, s.opacities,
                                                      s.sh_coeffs)]
    means, quats, scales, opac, sh = leaves
    out = torch.ops.splat200.project_views(means, quats, scales, opac, vm, full, Ks, s.width,
                                           s.height, 0.2, float("inf"), 0.0, sh, 3, campos,
                                           "radius")
    ref = stages.project_views(means.detach(), quats.detach(), scales.detach(), opac.detach(),
                               vm, full, Ks, s.width, s.height, 0.2, float("inf"), 0.0,
                               sh=sh.detach(), sh_degree=3, campos=campos,
                               normalize_quats=True)
    vis = ref.radii > 0
    assert torch.equal(out[3], ref.radii) and torch.equal(out[4], ref.tile_counts)
    assert torch.equal(out[0][vis], torch.stack(ref.centers)[vis])
    assert torch.equal(out[2], torch.stack(ref.colors))
    g = torch.Generator(device=d).manual_seed(2)
    w = [torch.randn(t.shape, device=d, generator=g) for t in out[:3]]
    (sum((t * wt).sum() for t, wt in zip(out[:3], w))).backward()
    want = torch.ops.splat200.project_views_backward(
        means.detach(), quats.detach(), scales.detach(), vm, full, Ks, s.width, s.height,
        out[3], sh.detach(), 3, campos, out[6], w[0], w[1], w[2])
    for leaf, wv in zip(leaves, want):
        assert rel_l2(leaf.grad.cpu(), wv.cpu()) <= 1e-6


def test_rade_ops_match_stage_api_and_autograd():
    """torch.ops.splat200.rade_* chained with autograd against rade.ops
    (prepare_gaussians -> bin_and_sort -> rasterize_to_pixels): the same five
    images and the same gradients (quaternions normalised once on each side:
    by F.normalize before the operators, in-kernel in rade.ops)."""
    from dsl_splat_b200 import PinholeCamera, rade

    d = torch.device("cuda", 0)
    s = make_scene(4, n=20000, width=320, height=240)
    W, H = s.width, s.height
    view, K = s.viewmats[0].to(d).contiguous(), s.Ks[0].to(d).contiguous()
    full, _, _ = torch.ops.splat200.cameras_prepare(view[None], K[None], W, H, True)
    g = torch.Generator().manual_seed(9)
    feats0 = torch.rand(s.means.shape[0], 35, generator=g).to(d)
    bg = torch.rand(35, generator=g).to(d)
    ups = [torch.randn(H, W, k, generator=g).to(d) for k in (35, 1, 1, 1, 3)]

    def leaves():
        out = [t.to(d).clone().requires_grad_(True)
               for t in (s.means, s.quats, s.scales, s.opacities, feats0)]
        return out

    a = leaves()
    ctr, con, radii, tiles, depths, planes, normals = torch.ops.splat200.rade_project(
        a[0], F.normalize(a[1], dim=-1), a[2], a[3], view, full[0], K, W, H, 0.2, float("inf"),
        0.0, 0.0)
    ranges, ids = torch.ops.splat200.bin_and_sort(ctr, con, radii, tiles, depths, W, H,
                                                  "radius")
    img_ops = torch.ops.splat200.rade_render(ctr, con, planes, normals, ranges, ids, a[4], bg, K,
                                             W, H)[:5]
    torch.autograd.backward(img_ops, ups)

    b = leaves()
    geo = rade.ops.prepare_gaussians(b[0], b[1], b[2], b[3], PinholeCamera(view, K, W, H, 0.2))
    px = rade.ops.rasterize_to_pixels(geo, rade.ops.bin_and_sort(geo), b[4], bg)
    img_api = (px.features, px.alpha, px.depth, px.median_depth, px.normals)
    torch.autograd.backward(img_api, ups)

    for x, y in zip(img_ops, img_api):
        assert (x - y).abs().max().item() <= 1e-5
    for x, y, name in zip(a, b, ("means", "quats", "scales", "opacities", "features")):
        assert rel_l2(x.grad.cpu().numpy(), y.grad.cpu().numpy()) <= 1e-4, name
