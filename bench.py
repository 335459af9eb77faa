#!/usr/bin/env python
"""Forward+backward frames/s of gs3d.rasterize on the BASELINE config-1 scene.

Workload: 1M Gaussians, SH3, one 1920x1080
pinhole camera per GPU, absgrad metadata, preallocated upstream image
gradients (the reference's benchmark convention, rade/README.md:194-196).
Seeded synthetic data with the config's distributions (no dataset).  The
Gaussians (236 MB/step of parameters and gradients) exceed the 126 MB L2,
so no extra L2 flush is done between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 is launched with torchrun, one rank per GPU: every rank renders its
own camera of the shared scene (weak scaling) and the per-Gaussian gradients
are summed with an NCCL all-reduce each step (the path's only exchange).
`--impl reference` times the reference algorithm's CPU restatement (the
oracle: dsl_splat's Warp code needs warp-lang, which is not installed) on
the host cores, without importing this package.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fwd+bwd frames/s, 3DGS SH3 1M Gaussians @1080p"
# other configs (parity cases, or --config 2 for the batched multi-view scene)
# report the same unit under their own name
CONFIG_METRICS = {2: "fwd+bwd frames/s (camera views), 3DGS SH3 3M Gaussians, 8 cameras "
                     "1296x840",
                  3: "fwd+bwd frames/s, AAA-Gaussians SH3 2M Gaussians @1080p",
                  4: "fwd+bwd frames/s, RaDe-GS SH3 1M Gaussians + 32 extra channels, depth/"
                     "median/normals @1600x1200"}
API_OF = {3: "aaa.rasterize", 4: "rade.rasterize"}


def metric_for(config: int) -> str:
    return CONFIG_METRICS.get(config, METRIC)
UNIT = "frames/s"
CHANNELS = 4  # RGB + the appended alpha column (gs3d/autograd.py:42-46)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", type=int, default=1)
    ap.add_argument("--buckets", type=int, default=1,
                    help="N > 1: Gaussian-range buckets of the gradient all-reduce (more "
                         "than one overlaps it with the projection backward; measured slower "
                         "on 2 B200s: 762 / 733 / 722 / 668 frames/s for 1 / 2 / 4 / 8)")
    ap.add_argument("--gaussians", type=int, default=None,
                    help="override the config's Gaussian count (smaller cases for ncu "
                         "captures; the bench line then names the reduced workload)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=15.0,
                    help="seconds of CPU work for the cpu_baseline sample")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def scenes_module():
    """dsl_splat_b200/scenes.py loaded by file path: the scene generator needs
    only torch, and loading it this way keeps the package __init__ (which maps
    libsplat200.so) out of the reference arm's process."""
    import importlib.util
    name = "_bench_scenes"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(
            name, os.path.join(ROOT, "dsl_splat_b200", "scenes.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


def workload(config: int, rank: int, world: int, gaussians: int | None = None):
    """The config scene.  Single-view configs: rank r looks from an orbit
    angle 2*pi*r/world (one view per rank).  Multi-view configs (config 2's
    8-camera batch): rank r renders the cameras k with k mod world == r
    (the round robin of sharding.local_cameras)."""
    sc = scenes_module()
    look_at, make_scene = sc.look_at, sc.make_scene
    s = make_scene(config, n=gaussians)
    cams = s.viewmats.shape[0]
    if cams > 1:
        idx = [k for k in range(cams) if k % world == rank]
        if not idx:
            raise SystemExit(f"config {config} has {cams} cameras: at most {cams} ranks")
        for name in ("viewmats", "Ks", "target", "grad_image", "grad_alpha"):
            setattr(s, name, getattr(s, name)[idx].contiguous())
        s.meta["cameras"] = cams
    elif world > 1 and rank > 0:
        th = 2.0 * math.pi * rank / world
        s.viewmats[0] = look_at(torch.tensor([8.0 * math.sin(th), 0.0, -8.0 * math.cos(th)]))
    return s


def describe(s, world):
    views = s.viewmats.shape[0]
    total = s.meta.get("cameras", world)
    api = API_OF.get(s.meta["config"], "gs3d.rasterize")
    extra = f" + {s.extras.shape[1]} extra channels" if s.extras is not None else ""
    return {
        "workload": f"config{s.meta['config']}: {api} SH{s.sh_degree} "
                    f"{s.means.shape[0]} Gaussians{extra} {s.width}x{s.height}, fwd+bwd, absgrad",
        "n_gaussians": int(s.means.shape[0]), "width": s.width, "height": s.height,
        "sh_degree": s.sh_degree, "views_per_gpu": views, "global_batch": total,
        "parallelism": f"camera-sharded dp{world}",
        "l2": "inputs larger than L2 (236 MB of Gaussian parameters+grads per step); no flush",
    }


# ---- clocks ------------------------------------------------------------------

class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        # nvidia-smi numbers GPUs physically; address ours by UUID instead of
        # the CUDA ordinal, which CUDA_VISIBLE_DEVICES may remap.
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:  # noqa: BLE001
            self.ident = str(device.index)
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.ident}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.file, stderr=subprocess.DEVNULL)
            # the timed region starts once the sampler has written its first
            # row (nvidia-smi can take longer to start than a short region)
            deadline = time.time() + 5.0
            while time.time() < deadline and os.path.getsize(self.file.name) == 0:
                time.sleep(0.02)
            self.start_rows = self._count_rows()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def _count_rows(self) -> int:
        with open(self.file.name) as f:
            return sum(1 for line in f if line.strip())

    def summary(self):
        self.file.flush()
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        # the rows written during the timed region (the ones before it only
        # showed that the sampler had started), unless the region was shorter
        # than one sampling interval
        start = getattr(self, "start_rows", 0)
        if len(rows) > start:
            rows = rows[start:]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4)
                          if len(r) > 5 + k and r[5 + k].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


# ---- CPU baseline (the oracle) ----------------------------------------------------

def cpu_band_step_rade(s, rows: int, y0: int = 0):
    """One RaDe-GS fwd+bwd of the oracle on image rows [y0, y0+rows) of view 0:
    camera prep, projection, SH, binning, geometry blend and its backward in
    the C++ restatement (OpenMP), the projection VJP as float64 Torch
    autograd (oracle/rade_vjp.py, Torch's host threads) and the SH backward."""
    from oracle import oracle as O
    from oracle import rade_vjp
    import torch.nn.functional as F
    W = s.width
    K = s.Ks[0].numpy().copy()
    K[1, 2] -= y0
    view = s.viewmats[0].numpy()
    means, scales, opac = s.means.numpy(), s.scales.numpy(), s.opacities.numpy()
    qn = F.normalize(s.quats, dim=-1).numpy()
    full, _, campos, _ = O.cameras_prepare(view[None], K[None], W, rows, True)
    geo = O.rade_project(means, qn, scales, opac, view, full[0], K, W, rows)
    dirs = means - campos[0]
    colors, active = O.sh_forward(s.sh_coeffs.numpy(), dirs, s.sh_degree, geo["radii"])
    feats = np.concatenate([colors, s.extras.numpy()], 1)
    offsets = np.cumsum(geo["tiles"]).astype(np.int32)
    _, ids, ranges = O.bin_and_sort(geo["centers"], geo["radii"], geo["depths"], offsets, W,
                                    rows)
    bg = np.zeros(feats.shape[1], np.float32)
    image, aux, contrib = O.rade_render(W, rows, ranges, ids, geo["centers"], geo["conics"],
                                        feats, bg, geo["planes"], geo["normals"], K)
    rng = np.random.default_rng(y0)
    ups = [rng.standard_normal((rows, W, k)).astype(np.float32)
           for k in (feats.shape[1], 1, 1, 1, 3)]
    g = O.rade_render_backward(W, rows, ranges, ids, geo["centers"], geo["conics"], feats, bg,
                               geo["planes"], geo["normals"], K, image, aux, contrib, *ups)
    rade_vjp.project_backward(means, qn, scales, opac, view, full[0], K, W, rows, geo["radii"],
                              g["centers"], g["conics"], g["planes"], g["normals"],
                              planes=geo["planes"])
    O.sh_backward(s.sh_coeffs.numpy(), dirs, s.sh_degree, geo["radii"], active,
                  g["features"][:, :3].astype(np.float32))


def aaa_lowered_camera(view, K, width: int, height: int, near: float = 0.01, far: float = 1e10):
    """aaa/cameras.py:78-121 on the host for one camera (the same Torch
    arithmetic as dsl_splat_b200.aaa.cameras, without importing the package):
    V^T and (P V)^T storage, the camera centre, tan(fov/2) and (cx, cy)."""
    fx, fy, cx, cy = float(K[0, 0]), float(K[1, 1]), float(K[0, 2]), float(K[1, 2])
    p = torch.zeros(4, 4, dtype=torch.float32)
    k = torch.as_tensor(K, dtype=torch.float32)
    p[0, 0] = 2 * k[0, 0] / width
    p[1, 1] = 2 * k[1, 1] / height
    p[0, 2] = 2 * k[0, 2] / width - 1
    p[1, 2] = 2 * k[1, 2] / height - 1
    p[2, 2] = far / (far - near)
    p[2, 3] = -far * near / (far - near)
    p[3, 2] = 1
    v = torch.as_tensor(view, dtype=torch.float32)
    full = (p @ v).T.contiguous().numpy()
    campos = torch.linalg.inv(v)[:3, 3].contiguous().numpy()
    return (v.T.contiguous().numpy(), full, campos, (width / (2 * fx), height / (2 * fy)),
            (cx, cy))


def cpu_band_step_aaa(s, rows: int, y0: int = 0):
    """One aaa.rasterize fwd+bwd of the oracle on image rows [y0, y0+rows) of
    view 0 (principal point shifted by y0): SH colours, preprocessing,
    remainder cull, key emission and sort, HIER blend and its replay, the
    preprocessing and camera adjoints and the SH backward."""
    from oracle import oracle as O
    import torch.nn.functional as F
    W = s.width
    K = s.Ks[0].numpy().copy()
    K[1, 2] -= y0
    vt, full, campos, tanfov, principal = aaa_lowered_camera(s.viewmats[0].numpy(), K, W, rows)
    means, scales, opac = s.means.numpy(), s.scales.numpy(), s.opacities.numpy()
    qn = F.normalize(s.quats, dim=-1).numpy()
    pre = O.aaa_preprocess(means, qn, scales, opac, vt, full, campos, W, rows, tanfov, principal)
    final = O.aaa_cull_remainder(pre, W, rows)
    dirs = means - campos
    colors, active = O.sh_forward(s.sh_coeffs.numpy(), dirs, s.sh_degree, final["radii"])
    feats = np.concatenate([colors, np.ones((len(means), 1), np.float32)], 1)
    _, keys, values = O.aaa_duplicate(pre, final["radii"], final["tiles"], W, rows)
    T = ((W + 15) // 16) * ((rows + 15) // 16)
    _, ids, ranges = O.aaa_sort(keys, values, T)
    bg = np.zeros(4, np.float32)
    image, final_t, _ = O.aaa_render(W, rows, ranges, ids, pre["transforms"], pre["opacity"],
                                     feats, bg)
    up = np.concatenate([s.grad_image[0, y0:y0 + rows].numpy(),
                         s.grad_alpha[0, y0:y0 + rows].numpy()], -1)
    g = O.aaa_render_backward(W, rows, ranges, ids, pre["transforms"], pre["opacity"], feats, bg,
                              image, final_t, np.moveaxis(up, -1, 0).copy(), screen=True,
                              absgrad=True)
    up_t, up_o = g["transforms"].astype(np.float32), g["opacity"].astype(np.float32)
    O.aaa_preprocess_backward(means, qn, scales, opac, final["radii"], vt, full, campos, W, rows,
                              np.float32(W / (2.0 * tanfov[0])), up_t, up_o)
    O.aaa_camera_backward(means, qn, scales, final["radii"], pre["opacity"], vt, full, campos, W,
                          rows, np.float32(max(W / (2 * tanfov[0]), rows / (2 * tanfov[1]))),
                          up_t, up_o, np.zeros(3 * len(means), np.float32))
    O.sh_backward(s.sh_coeffs.numpy(), dirs, s.sh_degree, final["radii"], active,
                  g["colors"][:, :3].astype(np.float32))


def cpu_band_step(s, rows: int, y0: int = 0):
    """One fwd+bwd of the oracle on image rows [y0, y0+rows) of view 0."""
    if s.meta["config"] == 4:
        return cpu_band_step_rade(s, rows, y0)
    if s.meta["config"] == 3:
        return cpu_band_step_aaa(s, rows, y0)
    from oracle import oracle as O
    import torch.nn.functional as F
    K = s.Ks[0].numpy().copy()
    K[1, 2] -= y0
    qn = F.normalize(s.quats, dim=-1).numpy()
    means = s.means.numpy()
    r, bg = O.gs3d_view_forward(means, qn, s.scales.numpy(), s.opacities.numpy(),
                                s.viewmats[0].numpy(), K, s.width, rows,
                                sh_coeffs=s.sh_coeffs.numpy(), sh_degree=s.sh_degree)
    up = np.concatenate([s.grad_image[0, y0:y0 + rows].numpy(),
                         s.grad_alpha[0, y0:y0 + rows].numpy()], -1)
    O.gs3d_view_backward(r, bg, means, qn, s.scales.numpy(), s.opacities.numpy(),
                         s.viewmats[0].numpy(), K, s.width, rows, up,
                         sh_coeffs=s.sh_coeffs.numpy(), sh_degree=s.sh_degree)


def cpu_sample_rows(s, budget_s: float) -> int:
    """Tile-aligned band height whose fwd+bwd takes about budget_s seconds."""
    probe = min(128, s.height)
    t0 = time.perf_counter()
    cpu_band_step(s, probe)
    dt = time.perf_counter() - t0
    rows = int(probe * budget_s / max(dt, 1e-3)) // 16 * 16
    return max(16, min(s.height, rows))


def cpu_baseline(s, budget_s: float, steps: int = 1):
    from oracle import oracle as O
    threads = O.num_threads()
    rows = cpu_sample_rows(s, budget_s)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        cpu_band_step(s, rows)
        times.append(time.perf_counter() - t0)
    frac = rows / s.height
    value = frac / statistics.median(times)
    return {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"oracle (C++ restatement, OpenMP {threads} threads) fwd+bwd of image rows "
                      f"0-{rows} of {s.height} ({frac:.3f} of a frame, all {s.means.shape[0]} "
                      f"Gaussians projected), {steps} step(s); value = frame fraction / time"}


def run_reference(args, rank, world):
    """--impl reference: the reference algorithm's CPU restatement on host cores."""
    if rank != 0:
        return
    s = workload(args.config, 0, 1)
    from oracle import oracle as O
    threads = O.num_threads()
    budget = max(2.0, 150.0 / max(1, args.steps + args.warmup))
    rows = cpu_sample_rows(s, budget)
    for _ in range(args.warmup):
        cpu_band_step(s, rows)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu_band_step(s, rows)
        times.append(time.perf_counter() - t0)
    frac = rows / s.height
    value = frac * len(times) / sum(times)
    what = {3: "AAA-Gaussians (HIER 64/8/4 blend and replay)",
            4: "RaDe-GS (projection VJP as float64 Torch autograd)"}.get(args.config, "gs3d")
    sample = (f"oracle (C++ restatement of dsl_splat {what}; the Warp reference needs "
              f"warp-lang, absent) with {threads} OpenMP threads, image rows 0-{rows} of "
              f"{s.height} ({frac:.3f} frame) per step; value = frame fraction / time")
    line = {"metric": metric_for(args.config), "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, BASELINE config distributions)", "impl": "reference",
            "config": describe(s, 1),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- GPU arm ----------------------------------------------------------------------

def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def profile_traffic(kernel: str, config: int = 1):
    """dram read+write bytes per launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_config{config}.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


def algorithmic_bytes(kernel: str, n: int, nv: int, m: int, pixels: int, c: int = CHANNELS):
    """Per-launch algorithmic bytes of the blend kernels (the survey's per-view model;
    RaDe-GS adds the 24-byte plane and normal rows per staged pair, the five
    geometry planes plus auxiliary and contributor planes per pixel)."""
    if kernel == "render_forward":
        return 4 * m + m * (24 + 4 * c) + pixels * (4 * c + 8)
    if kernel == "render_backward":
        return pixels * (4 * c + 8) + 4 * m + m * (24 + 4 * c) + n * (24 + 4 * c + 8)
    if kernel == "rade_render_forward":
        return 4 * m + m * (48 + 4 * c) + pixels * (4 * (c + 6) + 16)
    if kernel == "rade_render_backward":
        return (pixels * (4 * (c + 6) + 16 + 4 * (c + 6)) + 4 * m + m * (48 + 4 * c)
                + n * (24 + 4 * c + 8 + 24))
    # AAA HIER blend: per (tile, Gaussian) pair its id, 4x4 Gaussian-to-screen
    # transform and opacity (68 B) and its features; per pixel the image,
    # transmittance and count; the replay adds the upstream image and the
    # saved forward per pixel and writes the transform, opacity, feature and
    # screen gradients per Gaussian
    if kernel == "aaa_render_forward":
        return 4 * m + m * (68 + 4 * c) + pixels * (4 * c + 8)
    if kernel == "aaa_render_backward":
        return pixels * (8 * c + 4) + 4 * m + m * (68 + 4 * c) + n * (64 + 4 + 4 * c + 16)
    raise KeyError(kernel)


def main():
    args = parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if not torch.cuda.is_available():
        print(json.dumps({"metric": METRIC, "error": "no CUDA device"}))
        sys.exit(1)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    from dsl_splat_b200 import aaa, gs3d, rade, sharding, stages
    from dsl_splat_b200._native import lib
    if world > 1:
        import torch.distributed as dist
        sharding.init_process_group("nccl", timeout_s=180.0, device=dev)
        pg = dist

    s = workload(args.config, rank, world, args.gaussians)
    means = s.means.to(dev).requires_grad_(True)
    quats = s.quats.to(dev).requires_grad_(True)
    scales = s.scales.to(dev).requires_grad_(True)
    opac = s.opacities.to(dev).requires_grad_(True)
    sh = s.sh_coeffs.to(dev).requires_grad_(True)
    params = [means, quats, scales, opac, sh]
    viewmats, Ks = s.viewmats.to(dev), s.Ks.to(dev)
    gF, gA = s.grad_image.to(dev), s.grad_alpha.to(dev)
    W, H = s.width, s.height
    last = {}
    is_rade = args.config == 4
    is_aaa = args.config == 3
    if is_rade:
        # RaDe-GS: 32 extra channels blended with RGB and
        # seeded N(0,1) upstream gradients for depth, median depth and normals
        extras = s.extras.to(dev).requires_grad_(True)
        params.append(extras)
        gen = torch.Generator().manual_seed(4004)
        views0 = s.viewmats.shape[0]
        gE = (torch.randn(views0, H, W, extras.shape[1], generator=gen) * 1e-3).to(dev)
        gD, gM = (torch.randn(views0, H, W, 1, generator=gen).to(dev) for _ in range(2))
        gN = torch.randn(views0, H, W, 3, generator=gen).to(dev)

    def rasterize_view(vm, kk):
        if is_aaa:
            return aaa.rasterize(means, quats, scales, opac, vm, kk, W, H, sh_coeffs=sh,
                                 absgrad=True)
        if is_rade:
            return rade.rasterize(means, quats, scales, opac, vm, kk, W, H, sh_coeffs=sh,
                                  extra_features=extras, absgrad=True)
        return gs3d.rasterize(means, quats, scales, opac, vm, kk, W, H, sh_coeffs=sh,
                              absgrad=True)

    def outputs_and_grads(res):
        if is_rade:
            return ([res.features, res.extra_features, res.alpha, res.depth, res.median_depth,
                     res.normals], [gF, gE, gA, gD, gM, gN])
        return [res.features, res.alpha], [gF, gA]

    # N > 1 or several views per rank: the per-Gaussian gradients go through
    # sharding.GradientSync (one buffer per parameter that every local view
    # accumulates into, all-reduced in --buckets Gaussian ranges when N > 1)
    views = int(viewmats.shape[0])
    frames_per_step = int(s.meta.get("cameras", world))
    # RaDe-GS (config 4, one view per rank): its projection does not feed a
    # GradientSync, so N > 1 all-reduces the parameter gradients (extras
    # included) in one coalesced NCCL group after each backward
    sync = (sharding.GradientSync(means, quats, scales, opac, sh,
                                  group=dist.group.WORLD if pg is not None else None,
                                  buckets=args.buckets)
            if (pg is not None or views > 1) and not (is_rade or is_aaa) else None)

    def reduce_rade_grads():
        if (is_rade or is_aaa) and pg is not None:
            sharding.allreduce_parameter_grads(params, group=dist.group.WORLD)

    def step():
        for p in params:
            p.grad = None
        if sync is None:
            res = rasterize_view(viewmats, Ks)
            torch.autograd.backward(*outputs_and_grads(res))
            reduce_rade_grads()
        else:
            with sync:
                res = rasterize_view(viewmats, Ks)
                torch.autograd.backward(*outputs_and_grads(res))
            sync.wait()
        last["res"] = res

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(max(3, args.warmup)):
        step()
    barrier()
    stages.TIMERS = {}
    launches0 = lib.splat_launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        barrier()
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        barrier()
    timers, stages.TIMERS = stages.TIMERS, None
    launches = lib.splat_launch_count() - launches0
    # float32: every NCCL algorithm (NVLS included) reduces it; ms to 7 digits
    elapsed = torch.tensor([start.elapsed_time(end)], device=dev, dtype=torch.float32)
    if pg is not None:
        pg.all_reduce(elapsed, op=pg.ReduceOp.MAX)
    ms = float(elapsed.item())
    value = frames_per_step * args.steps / (ms / 1000.0)

    # live roofline of the dominant kernel over the timed region
    res = last["res"]
    radii = res.meta["radii"].amax(-1)
    nv = int((radii > 0).sum()) // views  # per view (one launch of each kernel)
    m = int(res.meta["tiles_per_gauss"].sum()) // views
    n = int(means.shape[0])
    durations = {k: statistics.mean(a.elapsed_time(b) for a, b in v) for k, v in timers.items()}
    kernel = max(durations, key=durations.get)
    channels = 3 + extras.shape[1] if is_rade else CHANNELS
    per_launch = algorithmic_bytes(kernel, n, nv, m, W * H, channels)
    achieved = per_launch / (durations[kernel] / 1000.0) / 1e9
    peak, peak_kind = measured_peak()
    roofline = {"bound": "hbm", "kernel": kernel, "achieved": achieved, "peak": peak,
                "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_kind,
                "traffic": profile_traffic(kernel, args.config),
                "algorithmic_bytes_per_launch": per_launch,
                "launch_ms": durations[kernel], "pairs": m, "visible": nv,
                "kernel_ms": durations,
                # the blend's issue-bound unit: alpha evaluations, counted as
                # 256 pixels per (tile, Gaussian) pair before early termination
                "alpha_evals": {"per_frame_upper": 256 * m,
                                "per_s_upper": 256.0 * m * value,
                                "note": "blend kernels are issue-bound, not HBM-bound"}}

    # end to end through the public API with host buffers each step
    e2e = None
    if not args.no_e2e:
        target_host = s.target.contiguous().pin_memory()
        view_host = s.viewmats.contiguous().pin_memory()
        k_host = s.Ks.contiguous().pin_memory()
        # step k's inputs are copied from pinned memory on a copy stream while
        # step k-1's loss and backward compute (double-buffered prefetch, as a
        # training loop's loader does; queued once step k-1's forward is, so
        # the copy does not overlap the latency-bound binning, where it
        # measured 3 % slower); every copy lies inside the timed region
        copy_stream = torch.cuda.Stream(dev)
        bufs = [(torch.empty_like(target_host, device=dev), torch.empty_like(view_host, device=dev),
                 torch.empty_like(k_host, device=dev)) for _ in range(2)]
        ready = [torch.cuda.Event() for _ in range(2)]
        # step k's loss is copied into pinned memory on the compute stream and
        # read by the host at step k+1 (after the copy's event), as a training
        # loop logs its loss, so the read does not stall the launch queue
        loss_host = [torch.empty((), dtype=torch.float32).pin_memory() for _ in range(2)]
        loss_copied = [torch.cuda.Event() for _ in range(2)]
        losses = []

        def prefetch(k):
            copy_stream.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(copy_stream):
                for dst, src in zip(bufs[k % 2], (target_host, view_host, k_host)):
                    dst.copy_(src, non_blocking=True)
                ready[k % 2].record(copy_stream)

        def e2e_step(k, last):
            for p in params:
                p.grad = None
            torch.cuda.current_stream(dev).wait_event(ready[k % 2])
            target, vm, kk = bufs[k % 2]
            def loss_of(r):
                loss = (r.features - target).abs().mean()
                if is_rade:  # the geometry outputs take part in the loss as well
                    loss = loss + 1e-2 * (r.depth.mean() + r.normals.abs().mean())
                return loss

            if sync is None:
                r = rasterize_view(vm, kk)
                if not last:
                    prefetch(k + 1)
                loss = loss_of(r)
                loss.backward()
                reduce_rade_grads()
            else:
                with sync:
                    r = rasterize_view(vm, kk)
                    if not last:
                        prefetch(k + 1)
                    loss = loss_of(r)
                    loss.backward()
                sync.wait()
            loss_host[k % 2].copy_(loss.detach(), non_blocking=True)
            loss_copied[k % 2].record()
            if k > 0:
                loss_copied[(k - 1) % 2].synchronize()
                losses.append(float(loss_host[(k - 1) % 2]))
            if last:
                loss_copied[k % 2].synchronize()
                losses.append(float(loss_host[k % 2]))

        prefetch(0)
        for k in range(2):
            e2e_step(k, k == 1)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        prefetch(0)
        for k in range(args.steps):
            e2e_step(k, k == args.steps - 1)
        e1.record()
        barrier()
        assert len(losses) == args.steps + 2 and all(math.isfinite(v) for v in losses)
        et = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float32)
        if pg is not None:
            pg.all_reduce(et, op=pg.ReduceOp.MAX)
        e2e = {"value": frames_per_step * args.steps / (float(et.item()) / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": target_host.numel() * 4 + view_host.numel() * 4
               + k_host.numel() * 4, "d2h_bytes_per_step": 4,
               "path": f"{'rade' if is_rade else 'aaa' if is_aaa else 'gs3d'}.rasterize + L1 loss "
                       "+ backward; target "
                       "image, viewmat, K copied "
                       "H2D from pinned memory every step (prefetched one step ahead on a copy "
                       "stream, during the previous step's loss and backward) and the loss copied "
                       "D2H into pinned memory every step, read by the host one step later"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(s, args.cpu_budget)

    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    if rank == 0:
        line = {"metric": metric_for(args.config), "value": value, "unit": UNIT,
                "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
                "higher_is_better": True,
                # config 2 splits a fixed batch of cameras over the ranks; the
                # single-view configs give every rank its own view
                "scaling": "strong" if s.meta.get("cameras", 1) > 1 else "weak",
                "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded, BASELINE config distributions)",
                "config": dict(describe(s, world), **(
                    {"gradient_allreduce": (
                        "NCCL, one coalesced all-reduce of the parameter gradients after "
                        "the backward" if is_rade else
                        f"NCCL, {args.buckets} Gaussian-range bucket(s)"
                        + (" overlapped with the projection backward"
                           if args.buckets > 1 else ""))}
                    if world > 1 else {})),
                "roofline": roofline, "cpu_baseline": cpu,
                "e2e": e2e, "gpu_launches": int(launches), "clocks": clocks.summary()}
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
