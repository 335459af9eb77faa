"""Seeded synthetic scenes with the shapes and distributions of the benchmark
configurations (no dataset is used; every tensor is generated on the CPU with
``torch.Generator().manual_seed(1000 + config)`` so that CPU checkers and the
GPU see identical bits).

Config 0: 10k Gaussians in a box in front of an identity camera, 256x256, SH0.
Config 1: 1M Gaussians from 64 isotropic clusters in a radius-5 ball, SH3,
          one 1920x1080 camera at distance 8 looking at the origin.
Config 2: 3M Gaussians (config-1 distributions), 8 cameras 1296x840 on a
          radius-6 orbit at height 1.
Config 3: 2M Gaussians (config-1 distributions), SH3, one 1920x1080 camera
          (the AAA-Gaussians benchmark, aaa.rasterize).
Config 4: 1M Gaussians, SH3, 1600x1200, 32 extra channels (RaDe-GS shapes).

Sampling order: means, log-scales, quats, opacity logits, colours/SH, extras,
target image, upstream gradients.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass
class Scene:
    means: torch.Tensor
    quats: torch.Tensor
    scales: torch.Tensor
    opacities: torch.Tensor
    viewmats: torch.Tensor
    Ks: torch.Tensor
    width: int
    height: int
    sh_coeffs: torch.Tensor | None = None
    sh_degree: int | None = None
    features: torch.Tensor | None = None
    extras: torch.Tensor | None = None
    target: torch.Tensor | None = None
    grad_image: torch.Tensor | None = None
    grad_alpha: torch.Tensor | None = None
    meta: dict = field(default_factory=dict)

    def to(self, device) -> "Scene":
        out = Scene(**{k: (v.to(device) if isinstance(v, torch.Tensor) else v)
                       for k, v in self.__dict__.items()})
        return out


def look_at(center: torch.Tensor, target: torch.Tensor | None = None) -> torch.Tensor:
    """OpenCV world-to-camera matrix: z forward, world up (0,-1,0)."""
    center = center.double()
    target = torch.zeros(3, dtype=torch.float64) if target is None else target.double()
    z = target - center
    z = z / z.norm()
    up = torch.tensor([0.0, -1.0, 0.0], dtype=torch.float64)
    x = torch.linalg.cross(z, up)
    x = x / x.norm()
    y = torch.linalg.cross(z, x)
    R = torch.stack([x, y, z])
    view = torch.eye(4, dtype=torch.float64)
    view[:3, :3] = R
    view[:3, 3] = -R @ center
    return view.float()


def intrinsics(fx: float, fy: float, cx: float, cy: float) -> torch.Tensor:
    return torch.tensor([[fx, 0.0, cx], [0.0, fy, cy], [0.0, 0.0, 1.0]], dtype=torch.float32)


def _unit_quats(g: torch.Generator, n: int) -> torch.Tensor:
    q = torch.randn(n, 4, generator=g)
    return q / q.norm(dim=-1, keepdim=True)


def _cluster_means(g: torch.Generator, n: int, clusters: int = 64, radius: float = 5.0,
                   sigma: float = 0.5) -> torch.Tensor:
    centres = torch.empty(0, 3)
    while len(centres) < clusters:
        cand = (torch.rand(4 * clusters, 3, generator=g) * 2.0 - 1.0) * radius
        centres = torch.cat([centres, cand[cand.norm(dim=-1) <= radius]])
    centres = centres[:clusters]
    which = torch.randint(0, clusters, (n,), generator=g)
    return centres[which] + sigma * torch.randn(n, 3, generator=g)


def make_scene(config: int, *, n: int | None = None, width: int | None = None,
               height: int | None = None, sh_degree: int | None = None,
               cameras: int | None = None, with_grads: bool = True) -> Scene:
    """Build configuration ``config`` (optionally resized for parity tests)."""
    g = torch.Generator().manual_seed(1000 + config)
    if config == 0:
        n = 10_000 if n is None else n
        width = 256 if width is None else width
        height = 256 if height is None else height
        deg = 0 if sh_degree is None else sh_degree
        xy = torch.rand(n, 2, generator=g) * 2.0 - 1.0
        z = torch.rand(n, 1, generator=g) * 4.0 + 2.0
        means = torch.cat([xy, z], dim=1)
        scales = torch.exp(torch.randn(n, 3, generator=g) * 0.5 - 4.5)
        quats = _unit_quats(g, n)
        opacities = torch.sigmoid(torch.randn(n, generator=g))
        f = width * 1.0
        viewmats = torch.eye(4)[None]
        Ks = intrinsics(f, f, width / 2, height / 2)[None]
    elif config in (1, 2, 3, 4):
        defaults = {1: (1_000_000, 1920, 1080, 1100.0, 1),
                    3: (2_000_000, 1920, 1080, 1100.0, 1),
                    2: (3_000_000, 1296, 840, 1000.0, 8),
                    4: (1_000_000, 1600, 1200, 1200.0, 1)}[config]
        n = defaults[0] if n is None else n
        width = defaults[1] if width is None else width
        height = defaults[2] if height is None else height
        focal = defaults[3] * width / defaults[1]
        cams = defaults[4] if cameras is None else cameras
        deg = 3 if sh_degree is None else sh_degree
        means = _cluster_means(g, n)
        scales = torch.exp(torch.randn(n, 3, generator=g) * 0.7 - 4.0)
        quats = _unit_quats(g, n)
        opacities = torch.sigmoid(torch.randn(n, generator=g))
        if config == 2:
            views = []
            for k in range(cams):
                th = 2.0 * math.pi * k / cams
                views.append(look_at(torch.tensor([6.0 * math.sin(th), -1.0, -6.0 * math.cos(th)])))
            viewmats = torch.stack(views)
        else:
            viewmats = torch.stack([look_at(torch.tensor([0.0, 0.0, -8.0]))] * cams)
        Ks = torch.stack([intrinsics(focal, focal, width / 2, height / 2)] * cams)
    else:
        raise ValueError(f"unknown scene config {config}")
    k = (deg + 1) ** 2
    sh = torch.empty(n, k, 3)
    sh[:, 0] = torch.rand(n, 3, generator=g)
    if k > 1:
        sh[:, 1:] = torch.randn(n, k - 1, 3, generator=g) * 0.1
    extras = torch.randn(n, 32, generator=g) if config == 4 else None
    c = viewmats.shape[0]
    target = torch.rand(c, height, width, 3, generator=g)
    grad_image = grad_alpha = None
    if with_grads:
        grad_image = torch.randn(c, height, width, 3, generator=g) * 1e-3
        grad_alpha = torch.randn(c, height, width, 1, generator=g) * 1e-3
    return Scene(means=means.float(), quats=quats.float(), scales=scales.float(),
                 opacities=opacities.float(), viewmats=viewmats.float(), Ks=Ks.float(),
                 width=width, height=height, sh_coeffs=sh, sh_degree=deg, extras=extras,
                 target=target, grad_image=grad_image, grad_alpha=grad_alpha,
                 meta={"config": config})
