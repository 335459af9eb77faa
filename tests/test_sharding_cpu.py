"""Camera sharding on CPU ranks (gloo, world size 2).

Each rank renders its cameras with the oracle (the CPU checker; the GPU path
is exercised by bench.py --gpus N), sums its view gradients, and the ranks
all-reduce with dsl_splat_b200.sharding.  The result must equal the sum over
all views computed in one process (gs3d/api.py's sequential loop), within
1e-6 relative L2 (float64 sums).  A second test makes one rank leave before
the all-reduce: the other must get an error from the process group's
timeout, not hang.
"""

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT, rel_l2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _view_grads(scene, c):
    import torch.nn.functional as F
    from oracle import oracle as O
    qn = F.normalize(scene.quats, dim=-1).numpy()
    r, bg = O.gs3d_view_forward(scene.means.numpy(), qn, scene.scales.numpy(),
                                scene.opacities.numpy(), scene.viewmats[c].numpy(),
                                scene.Ks[c].numpy(), scene.width, scene.height,
                                sh_coeffs=scene.sh_coeffs.numpy(), sh_degree=scene.sh_degree)
    up = np.concatenate([scene.grad_image[c].numpy(), scene.grad_alpha[c].numpy()], -1)
    g = O.gs3d_view_backward(r, bg, scene.means.numpy(), qn, scene.scales.numpy(),
                             scene.opacities.numpy(), scene.viewmats[c].numpy(),
                             scene.Ks[c].numpy(), scene.width, scene.height, up,
                             sh_coeffs=scene.sh_coeffs.numpy(), sh_degree=scene.sh_degree)
    return [torch.from_numpy(np.asarray(x, np.float64)) for x in
            (g.means, g.quats_n, g.scales, g.opacities, g.sh)]


def _scene():
    from dsl_splat_b200.scenes import make_scene
    return make_scene(2, n=3000, width=96, height=64, cameras=4)


def _rade_view_grads(scene, c):
    """One RaDe-GS view through the oracle: projection, SH colours + 5 extra
    channels, binning, geometry blend and its backward with seeded upstream
    images, the projection VJP (float64 autograd) and the SH backward.
    Returns float64 gradients of (means, normalised quats, scales,
    opacities, SH, extras)."""
    import torch.nn.functional as F
    from oracle import oracle as O
    from oracle import rade_vjp
    W, H = scene.width, scene.height
    means, scales, opac = scene.means.numpy(), scene.scales.numpy(), scene.opacities.numpy()
    qn = F.normalize(scene.quats, dim=-1).numpy()
    sh, deg = scene.sh_coeffs.numpy(), scene.sh_degree
    view, K = scene.viewmats[c].numpy(), scene.Ks[c].numpy()
    extras = np.random.default_rng(1).standard_normal((len(means), 5)).astype(np.float32)
    full, _, campos, _ = O.cameras_prepare(view[None], K[None], W, H, True)
    geo = O.rade_project(means, qn, scales, opac, view, full[0], K, W, H)
    dirs = means - campos[0]
    colors, active = O.sh_forward(sh, dirs, deg, geo["radii"])
    feats = np.concatenate([colors, extras], 1)
    offsets = np.cumsum(geo["tiles"]).astype(np.int32)
    _, ids, ranges = O.bin_and_sort(geo["centers"], geo["radii"], geo["depths"], offsets, W, H)
    bg = np.zeros(feats.shape[1], np.float32)
    image, aux, contrib = O.rade_render(W, H, ranges, ids, geo["centers"], geo["conics"], feats,
                                        bg, geo["planes"], geo["normals"], K)
    rng = np.random.default_rng(100 + c)
    ups = [rng.standard_normal((H, W, k)).astype(np.float32) for k in (8, 1, 1, 1, 3)]
    g = O.rade_render_backward(W, H, ranges, ids, geo["centers"], geo["conics"], feats, bg,
                               geo["planes"], geo["normals"], K, image, aux, contrib, *ups)
    pg = rade_vjp.project_backward(means, qn, scales, opac, view, full[0], K, W, H,
                                   geo["radii"], g["centers"], g["conics"], g["planes"],
                                   g["normals"], planes=geo["planes"])
    g_sh, g_dirs = O.sh_backward(sh, dirs, deg, geo["radii"], active,
                                 g["features"][:, :3].astype(np.float32))
    out = [pg[0] + g_dirs, pg[1], pg[2], pg[3], g_sh, g["features"][:, 3:]]
    return [torch.from_numpy(np.asarray(x, np.float64)) for x in out]


def _worker(rank, world, port, outdir, mode):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    from dsl_splat_b200 import sharding
    sharding.init_process_group("gloo", timeout_s=15.0)
    scene = _scene()
    if mode == "leave" and rank == 1:
        return  # leaves between steps, before joining the all-reduce
    idx = sharding.local_cameras(scene.viewmats.shape[0], rank, world)
    grads_of = _rade_view_grads if mode == "rade" else _view_grads
    total = None
    for c in idx:
        g = grads_of(scene, c)
        total = g if total is None else [a + b for a, b in zip(total, g)]
    status = "ok"
    try:
        sharding.allreduce_gradients(total)
    except Exception as e:  # noqa: BLE001 - the failure is the point
        status = f"error: {type(e).__name__}"
    torch.save({"grads": total, "idx": idx, "status": status},
               os.path.join(outdir, f"rank{rank}.pt"))
    if mode != "leave":
        dist.destroy_process_group()


def _run(world, mode, tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path), mode))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    return [torch.load(os.path.join(tmp_path, f"rank{r}.pt")) if
            os.path.exists(os.path.join(tmp_path, f"rank{r}.pt")) else None for r in range(world)]


def test_local_cameras_round_robin():
    from dsl_splat_b200.sharding import local_cameras
    assert local_cameras(8, 0, 2) == [0, 2, 4, 6]
    assert local_cameras(8, 3, 4) == [3, 7]
    assert sorted(sum((local_cameras(7, r, 3) for r in range(3)), [])) == list(range(7))
    with pytest.raises(ValueError):
        local_cameras(4, 2, 2)


def test_two_rank_allreduce_equals_sequential_sum(tmp_path):
    results = _run(2, "sum", tmp_path)
    scene = _scene()
    want = None
    for c in range(scene.viewmats.shape[0]):
        g = _view_grads(scene, c)
        want = g if want is None else [a + b for a, b in zip(want, g)]
    assert results[0]["idx"] == [0, 2] and results[1]["idx"] == [1, 3]
    for res in results:
        assert res["status"] == "ok"
        for got, ref in zip(res["grads"], want):
            assert rel_l2(got.numpy(), ref.numpy()) <= 1e-6


def test_two_rank_rade_allreduce_equals_sequential_sum(tmp_path):
    """The RaDe-GS view gradients (bench.py --config 4 at N > 1 all-reduces
    them after each backward) sharded over two gloo ranks."""
    results = _run(2, "rade", tmp_path)
    scene = _scene()
    want = None
    for c in range(scene.viewmats.shape[0]):
        g = _rade_view_grads(scene, c)
        want = g if want is None else [a + b for a, b in zip(want, g)]
    for res in results:
        assert res["status"] == "ok"
        for got, ref in zip(res["grads"], want):
            assert np.isfinite(ref.numpy()).all() and ref.abs().sum() > 0
            assert rel_l2(got.numpy(), ref.numpy()) <= 1e-6


def test_rank_that_leaves_is_detected_by_timeout(tmp_path):
    results = _run(2, "leave", tmp_path)
    assert results[1] is None
    assert results[0]["status"].startswith("error")


def _contribution(shape, rank, view, step):
    n = shape[0]
    base = torch.arange(n, dtype=torch.float32).reshape((n,) + (1,) * (len(shape) - 1))
    return (base + 1000.0 * rank + 100.0 * view + 10.0 * step).expand(shape).contiguous()


SYNC_SHAPES = [(101, 3), (101, 4), (101, 3), (101,), (101, 16, 3)]


def _zero_view_worker(rank, world, port, outdir, buckets):
    """One camera, two ranks: rank 0 renders the view (driven here as the
    projection backward drives GradientSync), rank 1 has no local view and
    only calls wait(); both must end with rank 0's gradients, and the
    plain all-reduce of parameter gradients must line up the same way."""
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    from dsl_splat_b200 import sharding
    sharding.init_process_group("gloo", timeout_s=30.0)
    assert sharding.local_cameras(1, rank, world) == ([0] if rank == 0 else [])
    params = [torch.zeros(s, requires_grad=True) for s in SYNC_SHAPES]
    sync = sharding.GradientSync(*params, group=dist.group.WORLD, buckets=buckets)
    with sync:
        if rank == 0:
            sync.register_view()
            bufs, _, last = sync.begin_view()
            for buf, shape in zip(bufs.values(), SYNC_SHAPES):
                buf.copy_(_contribution(shape, 0, 0, 0))
            for lo, hi in sharding.bucket_bounds(SYNC_SHAPES[0][0], sync.buckets):
                sync.reduce_range(lo, hi)
            sync.finish()
    sync.wait()
    plain = [torch.zeros(s, requires_grad=True) for s in SYNC_SHAPES]
    if rank == 0:
        for p, shape in zip(plain, SYNC_SHAPES):
            p.grad = _contribution(shape, 0, 1, 0)
    sharding.allreduce_parameter_grads(plain, group=dist.group.WORLD)
    torch.save({"sync": [p.grad.clone() for p in params],
                "plain": [p.grad.clone() for p in plain]},
               os.path.join(outdir, f"rank{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("buckets", [1, 3])
def test_rank_without_views_joins_reductions(tmp_path, buckets):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_zero_view_worker, args=(r, 2, port, str(tmp_path), buckets))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish (collectives did not line up)")
    for r in range(2):
        res = torch.load(os.path.join(tmp_path, f"rank{r}.pt"))
        for got, shape in zip(res["sync"], SYNC_SHAPES):
            assert torch.equal(got, _contribution(shape, 0, 0, 0))
        for got, shape in zip(res["plain"], SYNC_SHAPES):
            assert torch.equal(got, _contribution(shape, 0, 1, 0))


def _sync_worker(rank, world, port, outdir, buckets):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    from dsl_splat_b200 import sharding
    sharding.init_process_group("gloo", timeout_s=30.0)
    params = [torch.zeros(s, requires_grad=True) for s in SYNC_SHAPES]
    sync = sharding.GradientSync(*params, group=dist.group.WORLD, buckets=buckets)
    flags = []
    for step in range(2):  # the second step accumulates into the first's p.grad
        with sync:
            for _ in range(2):
                sync.register_view()
            for view in range(2):
                bufs, accumulate, last = sync.begin_view()
                flags.append((accumulate, last))
                for (name, buf), shape in zip(bufs.items(), SYNC_SHAPES):
                    g = _contribution(shape, rank, view, step)
                    if accumulate:
                        buf.add_(g)
                    else:
                        buf.copy_(g)
                if last:
                    for lo, hi in sharding.bucket_bounds(SYNC_SHAPES[0][0], sync.buckets):
                        sync.reduce_range(lo, hi)
                    sync.finish()
        sync.wait()
    torch.save({"grads": [p.grad.clone() for p in params], "flags": flags},
               os.path.join(outdir, f"rank{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("buckets", [1, 3])
def test_gradient_sync_buckets_equal_full_sum(tmp_path, buckets):
    """GradientSync with gloo ranks: per-view accumulation, the last view's
    all-reduce (one flat buffer for one bucket, row ranges for three), and
    p.grad accumulation across steps give the sum of every rank's and view's
    gradients."""
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_sync_worker, args=(r, 2, port, str(tmp_path), buckets))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    for r in range(2):
        res = torch.load(os.path.join(tmp_path, f"rank{r}.pt"))
        # each step: view 0 overwrites the step's buffers, view 1 accumulates
        # and reduces; step 1's reduced sum is added to step 0's p.grad
        assert res["flags"] == [(False, False), (True, True), (False, False), (True, True)]
        for got, shape in zip(res["grads"], SYNC_SHAPES):
            want = sum(_contribution(shape, rank, view, step)
                       for rank in range(2) for view in range(2) for step in range(2))
            assert torch.equal(got, want)


def test_bucket_bounds_and_incomplete_backward():
    from dsl_splat_b200.sharding import GradientSync, bucket_bounds
    for n in (0, 1, 31, 32, 33, 1000, 1_000_000):
        for b in (1, 3, 4, 7):
            ranges = bucket_bounds(n, b)
            assert len(ranges) <= b
            if not n:
                assert ranges == []
                continue
            assert [lo for lo, _ in ranges] == [0] + [hi for _, hi in ranges[:-1]]
            assert ranges[-1][1] == n and all(lo < hi for lo, hi in ranges)
            assert all(lo % 32 == 0 for lo, _ in ranges)
    params = [torch.zeros(s, requires_grad=True) for s in SYNC_SHAPES]
    sync = GradientSync(*params)
    with sync:
        sync.register_view()
        sync.register_view()
        sync.begin_view()  # the second view's backward never runs
    with pytest.raises(RuntimeError, match="1 of 2"):
        sync.wait()
    with sync:
        with pytest.raises(RuntimeError, match="nest"):
            with GradientSync(*params):
                pass
