"""GPU parity: the sm_100a kernels (through the C ABI) against the CPU oracle.

Tolerances:
  * integer outputs -- radii, tile counts, sorted ids, ranges, keys,
    contributor counts -- bit-exact;
  * float forward outputs of the projection and SH (same float32 operation
    sequence on both sides) -- bit-exact; final transmittance bit-exact;
  * rendered colour/alpha -- max-abs <= 1e-5;
  * gradients -- relative L2 <= 1e-3 (atomic summation order differs).
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import rel_l2
from dsl_splat_b200 import stages
from dsl_splat_b200.scenes import make_scene
from oracle import oracle as O

pytestmark = pytest.mark.gpu

IMG_TOL = 1e-5
GRAD_TOL = 1e-3

CASES = {
    "c0": dict(config=0),
    "c1_small": dict(config=1, n=20000, width=480, height=270),
    "c2_view": dict(config=2, n=30000, width=324, height=210, cameras=1),
}


def _scene(name):
    return make_scene(**CASES[name])


def _dev():
    return torch.device("cuda", 0)


class Prepared:
    """One view's inputs on the GPU plus the identical float32 arrays on the CPU."""

    def __init__(self, scene, view=0):
        d = _dev()
        self.s = scene
        self.W, self.H = scene.width, scene.height
        self.means = scene.means.to(d)
        self.quats = F.normalize(scene.quats.to(d), dim=-1)
        self.scales = scene.scales.to(d)
        self.opac = scene.opacities.to(d)
        self.view = scene.viewmats[view].to(d).contiguous()
        self.K = scene.Ks[view].to(d).contiguous()
        self.sh = scene.sh_coeffs.to(d)
        self.deg = scene.sh_degree
        full, inv, centers = stages.cameras_prepare(self.view[None], self.K[None], self.W, self.H,
                                                    self.deg > 0)
        self.full, self.inv = full[0], (inv[0] if self.deg > 0 else None)
        self.campos = centers[0] if self.deg > 0 else None
        self.np = {k: getattr(self, k).cpu().numpy() for k in
                   ("means", "quats", "scales", "opac", "view", "K", "sh", "full")}

    def project(self):
        return stages.project_fused(self.means, self.quats, self.scales, self.opac, self.view,
                                    self.full, self.K, self.W, self.H, 0.2, float("inf"), 0.0,
                                    sh=self.sh, sh_degree=self.deg, campos=self.campos)


def _oracle_view(p: Prepared):
    r, bg = O.gs3d_view_forward(p.np["means"], p.np["quats"], p.np["scales"], p.np["opac"],
                                p.np["view"], p.np["K"], p.W, p.H, sh_coeffs=p.np["sh"],
                                sh_degree=p.deg)
    return r, bg


@pytest.mark.parametrize("case", list(CASES))
def test_cameras_bit_exact(case):
    p = Prepared(_scene(case))
    full, inv, centers, err = O.cameras_prepare(p.np["view"][None], p.np["K"][None], p.W, p.H,
                                                True)
    g_full, g_inv, g_centers = stages.cameras_prepare(p.view[None], p.K[None], p.W, p.H, True)
    assert err[0] == 0
    np.testing.assert_array_equal(g_full.cpu().numpy(), full)
    np.testing.assert_array_equal(g_inv.cpu().numpy(), inv)
    np.testing.assert_array_equal(g_centers.cpu().numpy(), centers)
    gf = np.random.default_rng(0).standard_normal((1, 4, 4)).astype(np.float32)
    gc = np.random.default_rng(1).standard_normal((1, 3)).astype(np.float32)
    ref = O.cameras_backward(p.np["K"][None], gf, p.W, p.H, inv, gc)
    got = stages.cameras_backward(p.K[None], torch.from_numpy(gf).to(_dev()), p.W, p.H,
                                  g_inv, torch.from_numpy(gc).to(_dev()), (1, 4, 4))
    np.testing.assert_array_equal(got.cpu().numpy(), ref)


@pytest.mark.parametrize("case", list(CASES))
def test_projection_and_sh_bit_exact(case):
    p = Prepared(_scene(case))
    out = p.project()
    r, _ = _oracle_view(p)
    radii = out.state.radii.cpu().numpy()
    np.testing.assert_array_equal(radii, r.proj.radii)
    np.testing.assert_array_equal(out.state.tile_counts.cpu().numpy(), r.proj.tiles)
    vis = radii > 0
    assert vis.sum() > 0
    np.testing.assert_array_equal(out.state.centers.cpu().numpy()[vis], r.proj.centers[vis])
    np.testing.assert_array_equal(out.state.conics.cpu().numpy()[vis], r.proj.conics[vis])
    np.testing.assert_array_equal(out.state.depths.cpu().numpy()[vis], r.proj.depths[vis])
    np.testing.assert_array_equal(out.colors.cpu().numpy(), r.features[:, :3])
    np.testing.assert_array_equal(out.active.cpu().numpy(), r.colors_active)
    # dense metadata: visible rows copied, culled rows zero (metadata.py:12-31)
    m2d = out.means2d.cpu().numpy()
    np.testing.assert_array_equal(m2d[vis], r.proj.centers[vis])
    assert not m2d[~vis].any()
    np.testing.assert_array_equal(out.opacities.cpu().numpy()[vis], r.proj.conics[vis, 3])
    meta = stages.metadata(out.state)
    np.testing.assert_array_equal(meta["means2d"].cpu().numpy(), m2d)


@pytest.mark.parametrize("case", list(CASES))
def test_binning_bit_exact(case):
    p = Prepared(_scene(case))
    out = p.project()
    bins = stages.bin_and_sort(out.state, p.W, p.H)
    r, _ = _oracle_view(p)
    ranges = bins["ranges"].cpu().numpy()
    ids = bins["point_list"].cpu().numpy()
    np.testing.assert_array_equal(ranges, r.ranges)
    np.testing.assert_array_equal(ids, r.ids)
    # the 64-bit keys the reference sorts: (tile << 32) | float bits(depth)
    depth_bits = out.state.depths.cpu().numpy().view(np.uint32).astype(np.uint64)
    tile_of = np.repeat(np.arange(len(ranges), dtype=np.uint64), ranges[:, 1] - ranges[:, 0])
    keys = (tile_of << np.uint64(32)) | depth_bits[ids]
    np.testing.assert_array_equal(keys, r.keys)
    offsets, m = stages.scan_counts(out.state.tile_counts)
    ref_off, ref_m = O.scan_counts(r.proj.tiles)
    assert m == ref_m == len(ids)
    np.testing.assert_array_equal(offsets.cpu().numpy(), ref_off)


def _render_case(case):
    p = Prepared(_scene(case))
    out = p.project()
    bins = stages.bin_and_sort(out.state, p.W, p.H)
    r, bg = _oracle_view(p)
    return p, out, bins, r, bg


@pytest.mark.parametrize("case", list(CASES))
def test_render_forward(case):
    p, out, bins, r, bg = _render_case(case)
    bg_t = torch.from_numpy(bg).to(_dev())
    px = stages.render(out.state, bins, out.colors, None, True, bg_t, p.W, p.H)
    np.testing.assert_array_equal(px.contributors.cpu().numpy(), r.contributors)
    np.testing.assert_array_equal(px.transmittance.cpu().numpy(), r.final_t)
    img = np.moveaxis(px.features.cpu().numpy(), -1, 0)
    assert np.abs(img - r.image).max() <= IMG_TOL
    planar = stages.render(out.state, bins, out.colors, None, True, bg_t, p.W, p.H, planar=True)
    np.testing.assert_array_equal(planar.features.cpu().numpy(), img)


@pytest.mark.parametrize("case", list(CASES))
def test_render_backward(case):
    p, out, bins, r, bg = _render_case(case)
    bg_t = torch.from_numpy(bg).to(_dev())
    px = stages.render(out.state, bins, out.colors, None, True, bg_t, p.W, p.H)
    up = np.random.default_rng(7).standard_normal((p.H, p.W, 4)).astype(np.float32)
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
    assert not rf[:, 3].any()  # constant tail: no feature gradient for the ones column


@pytest.mark.parametrize("case", list(CASES))
def test_render_separate_alpha(case):
    """Colour and alpha in separate buffers (forward) and separate upstream
    gradients (backward) give the combined layout's values exactly."""
    p, out, bins, r, bg = _render_case(case)
    d = _dev()
    bg_t = torch.from_numpy(bg).to(d)
    px = stages.render(out.state, bins, out.colors, None, True, bg_t, p.W, p.H)
    sep = stages.render(out.state, bins, out.colors, None, True, bg_t, p.W, p.H,
                        separate_alpha=True)
    assert torch.equal(sep.features, px.features[..., :3])
    assert torch.equal(sep.alpha, px.features[..., 3:])
    assert torch.equal(sep.contributors, px.contributors)
    up = torch.from_numpy(np.random.default_rng(7).standard_normal((p.H, p.W, 4))
                          .astype(np.float32)).to(d)
    kw = dict(absgrad=True, constant_tail=1)
    whole = stages.render_backward(out.state, bins, out.colors, None, True, bg_t,
                                   px.transmittance, px.contributors, up, p.W, p.H, **kw)
    split = stages.render_backward(out.state, bins, out.colors, None, True, bg_t,
                                   px.transmittance, px.contributors, up[..., :3].contiguous(),
                                   p.W, p.H, gradient_alpha=up[..., 3:].contiguous(),
                                   separate_alpha=True, **kw)
    for a, b in zip(whole, split):
        if a is not None:
            assert rel_l2(b.cpu().numpy(), a.cpu().numpy()) <= 1e-5
    # a missing alpha gradient reads as zero, not as a neighbouring colour
    no_alpha = stages.render_backward(out.state, bins, out.colors, None, True, bg_t,
                                      px.transmittance, px.contributors,
                                      up[..., :3].contiguous(), p.W, p.H,
                                      separate_alpha=True, **kw)
    up0 = up.clone()
    up0[..., 3] = 0
    ref0 = stages.render_backward(out.state, bins, out.colors, None, True, bg_t,
                                  px.transmittance, px.contributors, up0, p.W, p.H, **kw)
    for a, b in zip(ref0, no_alpha):
        if a is not None:
            assert rel_l2(b.cpu().numpy(), a.cpu().numpy()) <= 1e-5


@pytest.mark.parametrize("case", list(CASES))
def test_projection_normalizes_raw_quaternions(case):
    """normalize_quats: the kernel's normalisation is bit-identical to Torch's
    CUDA F.normalize followed by the projection."""
    p = Prepared(_scene(case))
    d = _dev()
    raw = p.s.quats.to(d) * torch.linspace(1e-3, 40.0, len(p.means), device=d)[:, None]
    ref = stages.project_fused(p.means, F.normalize(raw, dim=-1), p.scales, p.opac, p.view,
                               p.full, p.K, p.W, p.H, 0.2, float("inf"), 0.0, sh=p.sh,
                               sh_degree=p.deg, campos=p.campos)
    got = stages.project_fused(p.means, raw, p.scales, p.opac, p.view, p.full, p.K, p.W, p.H,
                               0.2, float("inf"), 0.0, sh=p.sh, sh_degree=p.deg,
                               campos=p.campos, normalize_quats=True)
    assert torch.equal(got.state.radii, ref.state.radii)
    assert torch.equal(got.state.tile_counts, ref.state.tile_counts)
    # culled rows of centers/conics/depths are left unwritten, as the
    # reference's new_empty outputs are (gs3d/projection.py:324-328)
    vis = ref.state.radii > 0
    for name in ("centers", "conics", "depths"):
        assert torch.equal(getattr(got.state, name)[vis], getattr(ref.state, name)[vis]), name
    assert torch.equal(got.colors, ref.colors)


@pytest.mark.parametrize("case", list(CASES))
def test_projection_backward(case):
    p = Prepared(_scene(case))
    out = p.project()
    n = len(p.means)
    rng = np.random.default_rng(3)
    seed_c = rng.standard_normal((n, 2)).astype(np.float32)
    seed_q = (rng.standard_normal((n, 4)) * 1e-2).astype(np.float32)
    d = _dev()
    grads = stages.project_backward(p.means, p.quats, p.scales, p.opac, p.view, p.full, p.K, p.W,
                                    p.H, out.state, torch.from_numpy(seed_c).to(d),
                                    torch.from_numpy(seed_q).to(d), (True,) * 6)
    ref = O.project_backward(p.np["means"], p.np["quats"], p.np["scales"], p.np["opac"],
                             p.np["view"], p.np["full"], p.np["K"], p.W, p.H,
                             out.state.radii.cpu().numpy(), seed_c, seed_q)
    for got, want in zip(grads, ref):
        assert rel_l2(got.cpu().numpy(), want) <= GRAD_TOL


def _offset_copy(t: torch.Tensor, offset: int) -> torch.Tensor:
    """t copied into a buffer starting `offset` elements past an allocation
    (offset 1: 4-byte aligned only, which sends the kernel's staging of that
    input down its plain-copy path)."""
    flat = torch.zeros(t.numel() + 8, dtype=t.dtype, device=t.device)
    view = flat[offset:offset + t.numel()].view(t.shape)
    view.copy_(t)
    return view


FUSED_VARIANTS = [
    # degree, sh_k, camera grads, accumulate, misaligned inputs, raw quaternions
    (0, 1, False, False, False, False),
    (1, 4, True, False, True, False),
    (1, 16, False, False, False, True),
    (2, 9, False, True, True, False),
    (2, 16, True, True, False, True),
    (3, 16, True, False, False, True),
    (3, 16, False, True, True, False),
    (3, 20, False, False, False, False),
]


@pytest.mark.parametrize("deg,sh_k,camera,accumulate,misalign,raw", FUSED_VARIANTS)
def test_fused_projection_backward_variants(deg, sh_k, camera, accumulate, misalign, raw):
    """splat_project_backward_fused (projection VJP + SH VJP + normalisation
    VJP, staged per warp) against the oracle's projection and SH backward,
    over SH degrees, row strides, camera gradients, accumulation, a ragged
    last chunk and inputs without 16-byte alignment."""
    from dsl_splat_b200._native import check, lib, stream

    p = Prepared(_scene("c1_small"))
    out = p.project()
    d = _dev()
    n = len(p.means) - 13  # a partial last chunk of 32
    rng = np.random.default_rng(deg * 10 + sh_k)
    radii = out.state.radii[:n].contiguous()
    sh = torch.zeros((n, sh_k, 3), device=d)
    used = min(sh_k, 16)
    sh[:, :used] = p.sh[:n, :used]
    dirs = p.means[:n] - p.campos
    _, active = O.sh_forward(sh.cpu().numpy(), dirs.cpu().numpy(), deg, radii.cpu().numpy())
    seed_c = rng.standard_normal((n, 2)).astype(np.float32)
    seed_q = (rng.standard_normal((n, 4)) * 1e-2).astype(np.float32)
    seed_col = rng.standard_normal((n, 3)).astype(np.float32)
    quats_raw = (p.quats[:n] * torch.from_numpy(
        rng.uniform(0.5, 2.0, (n, 1)).astype(np.float32)).to(d)).contiguous()
    quats_n = F.normalize(quats_raw, dim=-1) if raw else p.quats[:n].contiguous()

    off = 1 if misalign else 0
    means = _offset_copy(p.means[:n], off)
    scales = _offset_copy(p.scales[:n], off)
    radii_in = _offset_copy(radii, off)
    sh_in = _offset_copy(sh, off)
    active_in = _offset_copy(torch.from_numpy(active).to(d), off)
    gcol = _offset_copy(torch.from_numpy(seed_col).to(d), off)
    prefill = {k: torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(d)
               for k, shape in (("m", (n, 3)), ("q", (n, 4)), ("s", (n, 3)), ("o", (n,)),
                                ("sh", (n, sh_k, 3)))}
    outs = {k: _offset_copy(v, off if k != "q" else 0) if accumulate
            else _offset_copy(torch.full_like(v, float("nan")), off if k != "q" else 0)
            for k, v in prefill.items()}
    cam = torch.zeros(35, device=d) if camera else None
    # held in names: a temporary freed inside the argument list would hand its
    # block to the next allocation
    seed_c_t, seed_q_t = torch.from_numpy(seed_c).to(d), torch.from_numpy(seed_q).to(d)
    check(lib.splat_project_backward_fused(
        n, means.data_ptr(), None if raw else quats_n.data_ptr(),
        quats_raw.data_ptr() if raw else None, scales.data_ptr(), p.view.data_ptr(),
        p.full.data_ptr(), p.K.data_ptr(), p.W, p.H, radii_in.data_ptr(),
        seed_c_t.data_ptr(), seed_q_t.data_ptr(),
        outs["m"].data_ptr(), outs["q"].data_ptr(), outs["s"].data_ptr(), outs["o"].data_ptr(),
        int(accumulate), None if cam is None else cam.data_ptr(), deg, sh_k,
        sh_in.data_ptr(), p.campos.data_ptr(), active_in.data_ptr(), gcol.data_ptr(), 3,
        outs["sh"].data_ptr(), stream(d)), "project_backward_fused")
    torch.cuda.synchronize(d)

    r_np = radii.cpu().numpy()
    gm, gq, gs, go, gv, gp = O.project_backward(
        p.np["means"][:n], quats_n.cpu().numpy(), p.np["scales"][:n], p.np["opac"][:n],
        p.np["view"], p.np["full"], p.np["K"], p.W, p.H, r_np, seed_c, seed_q)
    gsh, gdir = O.sh_backward(sh.cpu().numpy(), dirs.cpu().numpy(), deg, r_np, active, seed_col)
    if deg > 0:
        gm = gm + gdir
    if raw:
        x = quats_raw.cpu().requires_grad_(True)
        F.normalize(x, dim=-1).backward(torch.from_numpy(gq))
        gq = x.grad.numpy()
    want = {"m": gm, "q": gq, "s": gs, "o": go, "sh": gsh}
    for k, v in want.items():
        got = outs[k].cpu().numpy()
        if accumulate:
            got = got - prefill[k].cpu().numpy()
        assert np.isfinite(got).all(), k
        assert rel_l2(got, v) <= GRAD_TOL, k
    if camera:
        c = cam.cpu().numpy().astype(np.float64)
        assert rel_l2(c[:16].reshape(4, 4), gv) <= GRAD_TOL
        assert rel_l2(c[16:32].reshape(4, 4), gp) <= GRAD_TOL
        if deg > 0:
            assert rel_l2(c[32:35], -gdir.astype(np.float64).sum(0)) <= GRAD_TOL


@pytest.mark.parametrize("case", list(CASES))
def test_sh_standalone(case):
    p = Prepared(_scene(case))
    out = p.project()
    dirs = p.means - (p.campos if p.campos is not None else 0.0)
    colors, active = stages.sh_forward(p.sh, dirs, p.deg, out.state.radii, True)
    np.testing.assert_array_equal(colors.cpu().numpy(), out.colors.cpu().numpy())
    up = torch.randn(len(p.means), 3, device=_dev())
    gsh, gdir = stages.sh_backward(p.sh, dirs, p.deg, out.state.radii, active, up, True)
    rsh, rdir = O.sh_backward(p.np["sh"], dirs.cpu().numpy(), p.deg,
                              out.state.radii.cpu().numpy(), active.cpu().numpy(),
                              up.cpu().numpy(), need_dirs=True)
    assert rel_l2(gsh.cpu().numpy(), rsh) <= GRAD_TOL
    if p.deg > 0:
        assert rel_l2(gdir.cpu().numpy(), rdir) <= GRAD_TOL


def test_expf_matches_oracle_and_cuda():
    x = np.concatenate([np.linspace(-80.0, 0.0, 200001, dtype=np.float32),
                        np.float32(-np.logspace(-8, 1.9, 5001))]).astype(np.float32)
    d = _dev()
    xt = torch.from_numpy(x).to(d)
    ours = torch.empty_like(xt)
    cuda = torch.empty_like(xt)
    from dsl_splat_b200._native import check, lib, stream
    check(lib.splat_debug_expf(len(x), xt.data_ptr(), ours.data_ptr(), cuda.data_ptr(),
                               stream(d)), "debug_expf")
    ours, cuda = ours.cpu().numpy(), cuda.cpu().numpy()
    np.testing.assert_array_equal(ours, O.expf(x))
    # splat_expf returns 0 at and below -80 by design (alpha there is < 1e-34)
    live = x > -80.0
    assert not ours[~live].any()
    ulp = np.abs(ours[live].view(np.int32).astype(np.int64)
                 - cuda[live].view(np.int32).astype(np.int64))
    assert ulp.max() <= 3, ulp.max()


def test_empty_and_culled_scenes():
    d = _dev()
    s = make_scene(0, n=64)
    means = s.means.clone()
    means[:, 2] = -5.0  # all behind the camera
    W, H = s.width, s.height
    view, K = s.viewmats[0].to(d), s.Ks[0].to(d)
    full, _, _ = stages.cameras_prepare(view[None], K[None], W, H, False)
    st = stages.project(means.to(d), F.normalize(s.quats.to(d), dim=-1), s.scales.to(d),
                        s.opacities.to(d), view, full[0], K, W, H, 0.2, float("inf"), 0.0)
    assert int(st.radii.abs().sum()) == 0
    bins = stages.bin_and_sort(st, W, H)
    assert len(bins["point_list"]) == 0
    assert int(bins["ranges"].abs().sum()) == 0
    colors = torch.rand(64, 3, device=d)
    bg = torch.tensor([0.1, 0.2, 0.3, 0.0], device=d)
    px = stages.render(st, bins, colors, None, True, bg, W, H)
    assert torch.all(px.transmittance == 1)
    assert torch.allclose(px.features[..., :3], bg[:3].expand(H, W, 3))
    e = stages.project(means[:0].to(d), s.quats[:0].to(d), s.scales[:0].to(d),
                       s.opacities[:0].to(d), view, full[0], K, W, H, 0.2, float("inf"), 0.0)
    assert len(stages.bin_and_sort(e, W, H)["point_list"]) == 0


@pytest.mark.parametrize("width,height", [(1, 1), (17, 5), (3000, 2000), (4096, 4096),
                                          (4200, 4100)])
def test_tile_pass_counts(width, height):
    """Both binning paths vs the oracle: the chunked scatter (tile grids whose
    per-tile arrays fit in shared memory, incl. one above the 48 KB default)
    and the onesweep fallback with 2 and 3 tile-id passes (T <= 65536, > 65536)."""
    s = make_scene(0, n=3000, width=width, height=height)
    d = _dev()
    s.Ks[0] = torch.tensor([[width * 1.0, 0, width / 2], [0, width * 1.0, height / 2], [0, 0, 1]])
    view, K = s.viewmats[0].to(d), s.Ks[0].to(d)
    full, _, _ = stages.cameras_prepare(view[None], K[None], width, height, False)
    q = F.normalize(s.quats.to(d), dim=-1)
    st = stages.project(s.means.to(d), q, s.scales.to(d), s.opacities.to(d), view, full[0], K,
                        width, height, 0.2, float("inf"), 0.0)
    bins = stages.bin_and_sort(st, width, height)
    ref_p = O.project_forward(s.means.numpy(), q.cpu().numpy(), s.scales.numpy(),
                              s.opacities.numpy(), view.cpu().numpy(), full[0].cpu().numpy(),
                              K.cpu().numpy(), width, height)
    off, _ = O.scan_counts(ref_p.tiles)
    _, ids, ranges = O.bin_and_sort(ref_p.centers, ref_p.radii, ref_p.depths, off, width, height)
    np.testing.assert_array_equal(bins["ranges"].cpu().numpy(), ranges)
    np.testing.assert_array_equal(bins["point_list"].cpu().numpy(), ids)


@pytest.mark.parametrize("mode", ["snugbox", "accutile"])
@pytest.mark.parametrize("size", [(480, 270), (1, 1), (3000, 2000), (4096, 4096), (4200, 4100)])
def test_tile_modes_bit_exact(mode, size):
    """tile_mode snugbox/accutile: tile counts, point_list and ranges against
    the oracle; snugbox on the chunked scatter and (>40K tiles) the onesweep
    path, accutile on the strip emission with 1-3 tile-id passes; then the
    blend over those bins (contributors bit-exact)."""
    width, height = size
    s = make_scene(1, n=6000, width=width, height=height)
    d = _dev()
    s.Ks[0] = torch.tensor([[width * 0.9, 0, width / 2], [0, width * 0.9, height / 2], [0, 0, 1]])
    view, K = s.viewmats[0].to(d), s.Ks[0].to(d)
    full, _, _ = stages.cameras_prepare(view[None], K[None], width, height, False)
    q = F.normalize(s.quats.to(d), dim=-1)
    opac = s.opacities.clone()
    opac[::17] = 1.0 / 255.0 * (0.5 + torch.rand(len(opac[::17])))  # around the cut-off
    st = stages.project(s.means.to(d), q, s.scales.to(d), opac.to(d), view, full[0], K,
                        width, height, 0.2, float("inf"), 0.0, tile_mode=mode)
    ref = O.project_forward(s.means.numpy(), q.cpu().numpy(), s.scales.numpy(), opac.numpy(),
                            view.cpu().numpy(), full[0].cpu().numpy(), K.cpu().numpy(), width,
                            height, tile_mode=mode)
    np.testing.assert_array_equal(st.radii.cpu().numpy(), ref.radii)
    np.testing.assert_array_equal(st.tile_counts.cpu().numpy(), ref.tiles)
    bins = stages.bin_and_sort(st, width, height, tile_mode=mode)
    off, _ = O.scan_counts(ref.tiles)
    _, ids, ranges = O.bin_and_sort(ref.centers, ref.radii, ref.depths, off, width, height,
                                    conics=ref.conics, tile_mode=mode)
    np.testing.assert_array_equal(bins["ranges"].cpu().numpy(), ranges)
    np.testing.assert_array_equal(bins["point_list"].cpu().numpy(), ids)
    if width * height <= 480 * 270:
        feats = torch.rand(len(q), 3, device=d)
        bg = torch.zeros(4, device=d)
        px = stages.render(st, bins, feats, None, True, bg, width, height)
        attrs = np.concatenate([feats.cpu().numpy(), np.ones((len(q), 1), np.float32)], 1)
        _, _, contrib = O.render_forward(width, height, ranges, ids, ref.centers, ref.conics,
                                         attrs, np.zeros(4, np.float32))
        np.testing.assert_array_equal(px.contributors.cpu().numpy(), contrib)


def test_huge_footprint_and_out_of_view():
    """A Gaussian covering every tile, plus Gaussians outside the image."""
    d = _dev()
    s = make_scene(0, n=500)
    s.scales[0] = torch.tensor([2.0, 2.0, 2.0])
    s.means[0] = torch.tensor([0.0, 0.0, 3.0])
    s.means[1:50, 0] += 50.0  # far to the side
    p_scene = s
    p = Prepared(p_scene)
    out = p.project()
    bins = stages.bin_and_sort(out.state, p.W, p.H)
    r, bg = _oracle_view(p)
    np.testing.assert_array_equal(bins["point_list"].cpu().numpy(), r.ids)
    assert int(out.state.tile_counts[0]) == ((p.W + 15) // 16) * ((p.H + 15) // 16)
    px = stages.render(out.state, bins, out.colors, None, True, torch.from_numpy(bg).to(d), p.W,
                       p.H)
    np.testing.assert_array_equal(px.contributors.cpu().numpy(), r.contributors)


@pytest.mark.parametrize("deg,views", [(3, 4), (1, 2), (0, 3), (2, 17)])
def test_project_views_matches_per_view(deg, views):
    """splat_project_forward_views is bit-identical to one
    splat_project_forward_fused call per camera, and
    splat_project_backward_views equals the sum of the per-camera fused
    backwards (relative L2 1e-5); 17 cameras take two launches."""
    from dsl_splat_b200._native import check, lib, stream
    d = _dev()
    s = make_scene(2, n=20000 - 7, width=324, height=210, cameras=views)
    K = (deg + 1) ** 2
    means, scales, opac = s.means.to(d), s.scales.to(d), s.opacities.to(d)
    quats_raw = s.quats.to(d) * 1.7
    sh = s.sh_coeffs.to(d)[:, :K].contiguous()
    vm, Ks = s.viewmats.to(d), s.Ks.to(d)
    full, _, campos = stages.cameras_prepare(vm, Ks, s.width, s.height, True)
    campos = campos if deg > 0 else None
    args = (s.width, s.height, 0.2, float("inf"), 0.0)
    mv = stages.project_views(means, quats_raw, scales, opac, vm, full, Ks, *args, sh=sh,
                              sh_degree=deg, campos=campos, normalize_quats=True)
    singles = [stages.project_fused(means, quats_raw, scales, opac, vm[v], full[v], Ks[v], *args,
                                    sh=sh, sh_degree=deg,
                                    campos=None if campos is None else campos[v],
                                    normalize_quats=True) for v in range(views)]
    for v, one in enumerate(singles):
        vis = one.state.radii > 0
        assert torch.equal(mv.radii[v], one.state.radii)
        assert torch.equal(mv.tile_counts[v], one.state.tile_counts)
        assert torch.equal(mv.centers[v][vis], one.state.centers[vis])
        assert torch.equal(mv.conics[v][vis], one.state.conics[vis])
        assert torch.equal(mv.depths[v][vis], one.state.depths[vis])
        assert torch.equal(mv.colors[v], one.colors)
        assert torch.equal(mv.active[v], one.active)
        assert torch.equal(mv.means2d[v], one.means2d)
        assert torch.equal(mv.opacities[v], one.opacities)
        assert torch.equal(mv.conics3[v], one.conics3)

    n = len(means)
    g = torch.Generator(device=d).manual_seed(deg)
    gc = [torch.randn((n, 2), device=d, generator=g) for _ in range(views)]
    gq = [torch.randn((n, 4), device=d, generator=g) * 1e-2 for _ in range(views)]
    gcol = [torch.randn((n, 3), device=d, generator=g) for _ in range(views)]
    outs = [torch.empty_like(t) for t in (means, quats_raw, scales, opac, sh)]
    pin = stages.Args()
    check(lib.splat_project_backward_views(
        views, n, means.data_ptr(), None, quats_raw.data_ptr(), scales.data_ptr(),
        vm.data_ptr(), full.data_ptr(), Ks.data_ptr(), s.width, s.height,
        stages.pointer_table(mv.radii), stages.pointer_table(gc), stages.pointer_table(gq),
        *[o.data_ptr() for o in outs[:4]], 0, deg, K, sh.data_ptr(), pin(campos),
        stages.pointer_table(mv.active), stages.pointer_table(gcol), 3, outs[4].data_ptr(),
        stream(d)), "project_backward_views")
    want = [torch.zeros_like(o) for o in outs]
    for v in range(views):
        check(lib.splat_project_backward_fused(
            n, means.data_ptr(), None, quats_raw.data_ptr(), scales.data_ptr(),
            vm[v].data_ptr(), full[v].data_ptr(), Ks[v].data_ptr(), s.width, s.height,
            mv.radii[v].data_ptr(), gc[v].data_ptr(), gq[v].data_ptr(),
            *[w.data_ptr() for w in want[:4]], 1, None, deg, K, sh.data_ptr(),
            pin(None if campos is None else campos[v]), mv.active[v].data_ptr(),
            gcol[v].data_ptr(), 3, want[4].data_ptr(), stream(d)), "project_backward_fused")
    torch.cuda.synchronize(d)
    for name, o, w in zip(("means", "quats", "scales", "opacities", "sh"), outs, want):
        assert torch.isfinite(o).all(), name
        assert rel_l2(o.double().cpu().numpy(), w.double().cpu().numpy()) <= 1e-5, name


def test_tile_order_schedule():
    """splat_tile_order is a permutation of the tiles by descending pair
    count (within its 256 count buckets), and blending in that block order
    gives the same image, transmittance and contributors (bit for bit) and
    the same gradients as index order."""
    p = Prepared(_scene("c1_small"))
    out = p.project()
    bins = stages.bin_and_sort(out.state, p.W, p.H)
    order = stages.tile_order(bins).cpu().numpy()
    counts = (bins["ranges"][:, 1] - bins["ranges"][:, 0]).cpu().numpy()
    assert sorted(order.tolist()) == list(range(len(counts)))
    shift = max(0, int(counts.max()).bit_length() - 8)
    buckets = counts[order] >> shift
    assert (np.diff(buckets) <= 0).all()
    d = _dev()
    bg = torch.zeros(4, device=d)
    ref = stages.render(out.state, dict(ranges=bins["ranges"], point_list=bins["point_list"],
                                        tile_order=torch.arange(len(counts), dtype=torch.int32,
                                                                device=d)),
                        out.colors, None, True, bg, p.W, p.H)
    got = stages.render(out.state, bins, out.colors, None, True, bg, p.W, p.H)
    assert torch.equal(got.features, ref.features)
    assert torch.equal(got.transmittance, ref.transmittance)
    assert torch.equal(got.contributors, ref.contributors)
    up = torch.randn_like(got.features)
    g_ref = stages.render_backward(out.state, dict(ranges=bins["ranges"],
                                                   point_list=bins["point_list"],
                                                   tile_order=torch.arange(
                                                       len(counts), dtype=torch.int32, device=d)),
                                   out.colors, None, True, bg, ref.transmittance,
                                   ref.contributors, up, p.W, p.H, constant_tail=1)
    g_got = stages.render_backward(out.state, bins, out.colors, None, True, bg,
                                   got.transmittance, got.contributors, up, p.W, p.H,
                                   constant_tail=1)
    for a, b in zip(g_got[:3], g_ref[:3]):
        assert rel_l2(a.cpu().numpy(), b.cpu().numpy()) <= 1e-5


def test_early_emit_capacity_paths():
    """The chunked emit launched before the host reads the pair count (with
    the last call's count as capacity) gives the exact point list when the
    capacity fits, re-emits exactly when it is too small, and neither case
    records a device error."""
    from dsl_splat_b200._native import device_error
    p = Prepared(_scene("c1_small"))
    out = p.project()
    stages._PAIR_CAPACITY.clear()
    first = stages.bin_and_sort(out.state, p.W, p.H)          # no capacity yet: exact
    assert stages._PAIR_CAPACITY, "the chunked path records a capacity"
    again = stages.bin_and_sort(out.state, p.W, p.H)          # capacity fits
    assert torch.equal(again["point_list"], first["point_list"])
    assert torch.equal(again["ranges"], first["ranges"])
    for key in list(stages._PAIR_CAPACITY):
        stages._PAIR_CAPACITY[key] = 100                      # far too small
    small = stages.bin_and_sort(out.state, p.W, p.H)
    assert torch.equal(small["point_list"], first["point_list"])
    assert device_error(_dev()) == 0
