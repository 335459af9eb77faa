"""Float64 Torch autograd restatement of RaDe-GS's projection VJP (test
infrastructure only).

rade/projection.py:320-398 differentiates projection_loss (:294-317) with
Warp autodiff, except where the reference supplies custom adjoints:
adj_opacity_coefficient (:57-70), adj_reference_normalize (:78-84),
adj_invert_covariance (splatting/geometry.py:61-71) and
adj_reference_rotation (splatting/math.py:13-28).  Here the same loss is
written in Torch float64 with those four adjoints as autograd Functions;
everything else (clamp, normalize, max, sqrt, the plane and normal algebra)
is ordinary reverse mode, which is what Warp's autodiff computes.  Branches
(the minimum-scale axis, the degenerate-direction case) follow the float32
forward, decided from the float32 inputs.

This is the checker of the CUDA projection backward; the product never
imports it.
"""

from __future__ import annotations

import numpy as np
import torch


class _Rotation(torch.autograd.Function):
    """glm_rotation (primitives/math.py:33-45) with adj_reference_rotation."""

    @staticmethod
    def forward(ctx, q):
        ctx.save_for_backward(q)
        r, x, y, z = q.unbind(-1)
        rows = [[1 - 2 * (y * y + z * z), 2 * (x * y + r * z), 2 * (x * z - r * y)],
                [2 * (x * y - r * z), 1 - 2 * (x * x + z * z), 2 * (y * z + r * x)],
                [2 * (x * z + r * y), 2 * (y * z - r * x), 1 - 2 * (x * x + y * y)]]
        return torch.stack([torch.stack(row, -1) for row in rows], -2)

    @staticmethod
    def backward(ctx, g):
        (q,) = ctx.saved_tensors
        r, x, y, z = q.unbind(-1)

        def G(i, j):
            return g[..., i, j]

        return torch.stack([
            2 * (z * (G(0, 1) - G(1, 0)) + y * (G(2, 0) - G(0, 2)) + x * (G(1, 2) - G(2, 1))),
            2 * (y * (G(0, 1) + G(1, 0)) + z * (G(0, 2) + G(2, 0)) + r * (G(1, 2) - G(2, 1)))
            - 4 * x * (G(1, 1) + G(2, 2)),
            2 * (x * (G(0, 1) + G(1, 0)) + r * (G(2, 0) - G(0, 2)) + z * (G(1, 2) + G(2, 1)))
            - 4 * y * (G(0, 0) + G(2, 2)),
            2 * (r * (G(0, 1) - G(1, 0)) + x * (G(0, 2) + G(2, 0)) + y * (G(1, 2) + G(2, 1)))
            - 4 * z * (G(0, 0) + G(1, 1))], -1)


class _Inverse(torch.autograd.Function):
    """invert_covariance with adj_invert_covariance."""

    @staticmethod
    def forward(ctx, cov):
        ctx.save_for_backward(cov)
        a, b, c = cov.unbind(-1)
        inv = 1.0 / (a * c - b * b)
        return torch.stack([c * inv, -b * inv, a * inv], -1)

    @staticmethod
    def backward(ctx, g):
        (cov,) = ctx.saved_tensors
        a, b, c = cov.unbind(-1)
        det = a * c - b * b
        f = 1.0 / (det * det + 1e-7)
        x, y, z = g.unbind(-1)
        return f[:, None] * torch.stack([
            -c * c * x + b * c * y + (det - a * c) * z,
            2 * b * c * x - (det + 2 * b * b) * y + 2 * a * b * z,
            -a * a * z + a * b * y + (det - a * c) * x], -1)


class _OpacityCoefficient(torch.autograd.Function):
    """opacity_coefficient with adj_opacity_coefficient (rade/projection.py:50-70)."""

    @staticmethod
    def forward(ctx, cov, kernel: float):
        a, b, c = cov.unbind(-1)
        det0 = torch.clamp_min(a * c - b * b, 1e-6)
        det1 = torch.clamp_min((a + kernel) * (c + kernel) - b * b, 1e-6)
        coef = torch.sqrt(det0 / det1)
        ctx.save_for_backward(cov, det1, coef)
        ctx.kernel = kernel
        return coef

    @staticmethod
    def backward(ctx, g):
        cov, det1, coef = ctx.saved_tensors
        k = ctx.kernel
        a, b, c = cov.unbind(-1)
        d0 = g * 0.5 / (coef + 1e-6) / det1
        d1 = -d0 * coef
        return torch.stack([d0 * c + d1 * (c + k), -2.0 * b * (d0 + d1),
                            d0 * a + d1 * (a + k)], -1), None


class _ReferenceNormalize(torch.autograd.Function):
    """normalize with adj_reference_normalize (rade/projection.py:73-84): the
    VJP divides by the normalised vector's length."""

    @staticmethod
    def forward(ctx, v):
        n = v / v.norm(dim=-1, keepdim=True)
        ctx.save_for_backward(n)
        return n

    @staticmethod
    def backward(ctx, g):
        (n,) = ctx.saved_tensors
        return (g - n * (n * g).sum(-1, keepdim=True)) / n.norm(dim=-1, keepdim=True)


def _mv(m, v):
    return (m @ v[..., None])[..., 0]


def projection_loss(means, quats, scales, opac, view, proj, K, W, H, kernel_size, seeds,
                    scales32):
    """rade/projection.py:294-317 for the rows given (all visible).  seeds:
    (centers (n,2), conics (n,4), planes (n,3), normals (n,3)) float64;
    scales32: the float32 scales that decide the minimum-axis branch."""
    fx, fy = K[0, 0], K[1, 1]
    pos = means @ view[:3, :3].T + view[:3, 3]
    limx, limy = 1.3 * W / (2 * fx), 1.3 * H / (2 * fy)
    x, y, z = pos[:, 0] / pos[:, 2], pos[:, 1] / pos[:, 2], pos[:, 2]
    t0 = x.clamp(-limx, limx) * z
    t1 = y.clamp(-limy, limy) * z
    u, v = t0 / z, t1 / z
    R = _Rotation.apply(quats)
    camera = view[:3, :3].T
    zero = torch.zeros_like(z)
    J = torch.stack([torch.stack([fx / z, zero, zero], -1),
                     torch.stack([zero, fy / z, zero], -1),
                     torch.stack([-fx * t0 / (z * z), -fy * t1 / (z * z), zero], -1)], -2)
    transform = camera @ J
    M = (scales[:, :, None] * R) @ transform
    cov_m = M.transpose(1, 2) @ M
    cov = torch.stack([cov_m[:, 0, 0], cov_m[:, 1, 0], cov_m[:, 1, 1]], -1)
    # minimum axis (find_min_from_triple's ties), from the float32 scales
    s32 = np.asarray(scales32, np.float32)
    bigger = (s32[:, 0] < s32[:, 1]).astype(np.int64)
    i0, i1 = (bigger + 1) % 3, (bigger + 2) % 3
    rows = np.arange(len(s32))
    minimum = np.where(s32[rows, i0] > s32[rows, i1], i1, i0)
    full_rank = torch.from_numpy(s32[rows, minimum] > np.float32(1e-7))
    inv_m = ((1.0 / scales)[:, :, None] * R) @ camera
    ic_full = inv_m.transpose(1, 2) @ inv_m
    axis = R[torch.from_numpy(rows), torch.from_numpy(minimum)]
    ac = _mv(camera.T.expand(len(axis), 3, 3), axis)
    ic_flat = ac[:, :, None] * ac[:, None, :]
    ic = torch.where(full_rank[:, None, None], ic_full, ic_flat)
    uvh = torch.stack([u, v, torch.ones_like(u)], -1)
    d = _mv(ic, uvh)
    direction = d / d.norm(dim=-1, keepdim=True)
    length = torch.stack([t0, t1, z], -1).norm(dim=-1)
    factor = length / (u * u + v * v + 1.0)
    dot = (direction * uvh).sum(-1)
    denom = torch.where(dot > 1e-7, dot, torch.full_like(dot, 1e-7))
    dd = direction / denom[:, None]
    pl0 = (v * v + 1) * dd[:, 0] - u * v * dd[:, 1] - u * dd[:, 2]
    pl1 = -u * v * dd[:, 0] + (u * u + 1) * dd[:, 1] - v * dd[:, 2]
    plane = torch.stack([pl0 * factor / fx, pl1 * factor / fy, pos.norm(dim=-1)], -1)
    rn = torch.stack([-pl0 * factor, -pl1 * factor, -torch.ones_like(pl0)], -1)
    NJ = torch.stack([torch.stack([1 / z, zero, t0 / length], -1),
                      torch.stack([zero, 1 / z, t1 / length], -1),
                      torch.stack([-t0 / (z * z), -t1 / (z * z), z / length], -1)], -2)
    normal = _ReferenceNormalize.apply(_mv(NJ, rn))
    dilated = cov + torch.tensor([kernel_size, 0.0, kernel_size], dtype=cov.dtype)
    conic3 = _Inverse.apply(dilated)
    conic = torch.cat([conic3, (opac * _OpacityCoefficient.apply(cov, kernel_size))[:, None]], -1)
    clip = means @ proj[:, :3].T + proj[:, 3]
    inv_w = 1.0 / (clip[:, 3] + 1e-7)
    center = torch.stack([((clip[:, 0] * inv_w + 1) * W - 1) * 0.5,
                          ((clip[:, 1] * inv_w + 1) * H - 1) * 0.5], -1)
    seed_c, seed_q, seed_p, seed_n = seeds
    return ((center * seed_c).sum() + (conic * seed_q).sum() + (plane * seed_p).sum()
            + (normal * seed_n).sum())


def project_backward(means, quats, scales, opacities, view, proj, K, width, height, radii,
                     seed_centers, seed_conics, seed_planes, seed_normals, kernel_size=0.0,
                     planes=None):
    """Gradients (means, quats, scales, opacities, view, proj) as float64
    numpy arrays; culled rows zero.  planes: the forward's ray planes -- rows
    whose plane is all zero took the degenerate-direction branch, where the
    plane and normal are constants (their seeds are then dropped)."""
    vis = np.asarray(radii) > 0
    if planes is not None:
        flat = ~np.asarray(planes, np.float32).any(1)
    else:
        flat = np.zeros(len(vis), bool)

    def t(a, grad=False):
        return torch.tensor(np.asarray(a, np.float64), requires_grad=grad)

    leaves = [t(np.asarray(a)[vis], True) for a in (means, quats, scales, opacities)]
    view_t, proj_t = t(view, True), t(proj, True)
    keep = (~flat[vis]).astype(np.float64)[:, None]
    seeds = (t(np.asarray(seed_centers)[vis]), t(np.asarray(seed_conics)[vis]),
             t(np.asarray(seed_planes)[vis] * keep), t(np.asarray(seed_normals)[vis] * keep))
    loss = projection_loss(*leaves, view_t, proj_t, t(K), width, height, float(kernel_size),
                           seeds, np.asarray(scales, np.float32)[vis])
    loss.backward()
    out = []
    for leaf, full in zip(leaves, (means, quats, scales, opacities)):
        g = np.zeros(np.asarray(full).shape, np.float64)
        g[vis] = leaf.grad.numpy()
        out.append(g)
    return out + [view_t.grad.numpy(), proj_t.grad.numpy()]
