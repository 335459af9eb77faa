"""torch.ops.splat200.*: registration, schemas and fake (shape) kernels.

No GPU needed: fake CUDA tensors carry shapes and dtypes only, so this is
what torch.compile / torch.export see when they trace the stages.
"""

import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.symbolic_shapes import ShapeEnv

import dsl_splat_b200  # noqa: F401  (registers the operators)
from dsl_splat_b200.torch_ops import OPERATORS


def test_operators_registered_with_schemas():
    for name in OPERATORS:
        op = getattr(torch.ops.splat200, name)
        schema = str(op.default._schema)
        assert schema.startswith(f"splat200::{name}("), schema


def test_fake_shapes():
    n, W, H, C = 1000, 100, 60, 3
    with FakeTensorMode(shape_env=ShapeEnv()):
        dev = "cuda"
        f32 = dict(device=dev, dtype=torch.float32)
        means, quats = torch.empty(n, 3, **f32), torch.empty(n, 4, **f32)
        scales, opac = torch.empty(n, 3, **f32), torch.empty(n, **f32)
        view, K = torch.empty(4, 4, **f32), torch.empty(3, 3, **f32)
        full, inverse, centers_cam = torch.ops.splat200.cameras_prepare(view[None], K[None], W,
                                                                        H, True)
        assert full.shape == (1, 4, 4) and inverse.shape == (1, 4, 4)
        assert centers_cam.shape == (1, 3)
        ctr, con, radii, tiles, depths = torch.ops.splat200.project(
            means, quats, scales, opac, view, full[0], K, W, H, 0.2, float("inf"), 0.0,
            "snugbox")
        assert ctr.shape == (n, 2) and con.shape == (n, 4) and depths.shape == (n,)
        assert radii.dtype == tiles.dtype == torch.int32
        ranges, ids = torch.ops.splat200.bin_and_sort(ctr, con, radii, tiles, depths, W, H,
                                                      "radius")
        assert ranges.shape == (((W + 15) // 16) * ((H + 15) // 16), 2)
        assert ids.dim() == 1 and not isinstance(ids.shape[0], int)  # data-dependent size
        feats = torch.empty(n, C, **f32)
        image, alpha, final_t, contrib = torch.ops.splat200.render(
            ctr, con, ranges, ids, feats, torch.empty(C + 1, **f32), W, H)
        assert image.shape == (H, W, C) and alpha.shape == (H, W, 1)
        assert final_t.shape == (H, W) and contrib.dtype == torch.int32
        gc, gq, gf, gabs = torch.ops.splat200.render_backward(
            ctr, con, ranges, ids, feats, torch.empty(C + 1, **f32), final_t, contrib, image,
            alpha, W, H)
        assert gc.shape == (n, 2) and gq.shape == (n, 4) and gf.shape == (n, C)
        grads = torch.ops.splat200.project_backward(means, quats, scales, opac, view, full[0], K,
                                                    W, H, ctr, con, radii, tiles, depths, gc, gq)
        assert [tuple(g.shape) for g in grads] == [(n, 3), (n, 4), (n, 3), (n,), (4, 4), (4, 4)]
        coeffs, dirs = torch.empty(n, 16, 3, **f32), torch.empty(n, 3, **f32)
        colors, active = torch.ops.splat200.sh_forward(coeffs, dirs, 3, radii)
        assert colors.shape == (n, 3) and active.dtype == torch.uint8
        g_coeffs, g_dirs = torch.ops.splat200.sh_backward(coeffs, dirs, 3, radii, active, colors)
        assert g_coeffs.shape == coeffs.shape and g_dirs.shape == (n, 3)
        V = 3
        views, fulls, Ks = (torch.empty(V, 4, 4, **f32), torch.empty(V, 4, 4, **f32),
                            torch.empty(V, 3, 3, **f32))
        campos = torch.empty(V, 3, **f32)
        out = torch.ops.splat200.project_views(means, quats, scales, opac, views, fulls, Ks, W,
                                               H, 0.2, float("inf"), 0.0, coeffs, 3, campos,
                                               "radius")
        assert [tuple(t.shape) for t in out] == [(V, n, 2), (V, n, 4), (V, n, 3), (V, n),
                                                 (V, n), (V, n), (V, n, 3)]
        grads = torch.ops.splat200.project_views_backward(
            means, quats, scales, views, fulls, Ks, W, H, out[3], coeffs, 3, campos, out[6],
            out[0], out[1], out[2])
        assert [tuple(g.shape) for g in grads] == [(n, 3), (n, 4), (n, 3), (n,), (n, 16, 3)]


def test_rade_fake_shapes():
    n, W, H, C = 500, 64, 48, 7
    with FakeTensorMode(shape_env=ShapeEnv()):
        f32 = dict(device="cuda", dtype=torch.float32)
        means, quats = torch.empty(n, 3, **f32), torch.empty(n, 4, **f32)
        scales, opac = torch.empty(n, 3, **f32), torch.empty(n, **f32)
        view, full, K = torch.empty(4, 4, **f32), torch.empty(4, 4, **f32), torch.empty(3, 3, **f32)
        out = torch.ops.splat200.rade_project(means, quats, scales, opac, view, full, K, W, H,
                                              0.2, float("inf"), 0.0, 0.3)
        assert [tuple(t.shape) for t in out] == [(n, 2), (n, 4), (n,), (n,), (n,), (n, 3),
                                                 (n, 3)]
        ctr, con, radii, tiles, depths, planes, normals = out
        ranges, ids = torch.ops.splat200.bin_and_sort(ctr, con, radii, tiles, depths, W, H,
                                                      "radius")
        feats, bg = torch.empty(n, C, **f32), torch.empty(C, **f32)
        img = torch.ops.splat200.rade_render(ctr, con, planes, normals, ranges, ids, feats, bg,
                                             K, W, H)
        assert [tuple(t.shape) for t in img] == [(H, W, C), (H, W, 1), (H, W, 1), (H, W, 1),
                                                 (H, W, 3), (2, H, W), (2, H, W)]
        assert img[6].dtype == torch.int32
        g = torch.ops.splat200.rade_render_backward(ctr, con, planes, normals, ranges, ids,
                                                    feats, bg, K, img[1], img[4], img[5],
                                                    img[6], *img[:5], W, H)
        assert [tuple(t.shape) for t in g] == [(n, 2), (n, 4), (n, 3), (n, 3), (n, C), (n, 2)]
        pg = torch.ops.splat200.rade_project_backward(means, quats, scales, opac, view, full,
                                                      K, W, H, 0.3, radii, g[0], g[1], g[2],
                                                      g[3])
        assert [tuple(t.shape) for t in pg] == [(n, 3), (n, 4), (n, 3), (n,), (4, 4), (4, 4)]
