"""GradientSync on the GPU: gradients through gs3d.rasterize with the
per-view accumulation and the bucketed, overlapped all-reduce equal the
autograd path (relative L2 1e-5: only the summation order of the views
differs).

One-GPU cases run without a process group and with a one-rank NCCL group;
the multi-GPU case (skipped below two GPUs) spawns one NCCL rank per GPU,
each rendering the cameras k mod world, and compares every rank's gradients
with all cameras rendered on one GPU.
"""

import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT, rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-5
NAMES = ("means", "quats", "scales", "opacities", "sh")


def _scene():
    from dsl_splat_b200.scenes import make_scene
    return make_scene(2, n=30000, width=324, height=210, cameras=4)


def _leaves(s, dev):
    return [t.to(dev).requires_grad_(True) for t in
            (s.means, s.quats, s.scales, s.opacities, s.sh_coeffs)]


def _step(s, leaves, cams, dev, sync=None):
    from dsl_splat_b200 import gs3d
    means, quats, scales, opac, sh = leaves
    views = s.viewmats[cams].to(dev).requires_grad_(True)
    Ks = s.Ks[cams].to(dev)

    def run():
        res = gs3d.rasterize(means, quats, scales, opac, views, Ks, s.width, s.height,
                             sh_coeffs=sh, absgrad=True)
        torch.autograd.backward([res.features, res.alpha],
                                [s.grad_image[cams].to(dev), s.grad_alpha[cams].to(dev)])

    if sync is None:
        run()
    else:
        with sync:
            run()
        sync.wait()
    torch.cuda.synchronize(dev)
    return [p.grad.detach().clone() for p in leaves], views.grad.detach().clone()


def _compare(got, want):
    for name, g, w in zip(NAMES, got, want):
        assert rel_l2(g.double().cpu().numpy(), w.double().cpu().numpy()) <= TOL, name


def test_gradient_sync_matches_autograd_one_gpu():
    from dsl_splat_b200.sharding import GradientSync
    dev = torch.device("cuda", 0)
    s = _scene()
    cams = [0, 1, 2]
    want, want_views = _step(s, _leaves(s, dev), cams, dev)
    leaves = _leaves(s, dev)
    got, got_views = _step(s, leaves, cams, dev, GradientSync(*leaves, buckets=3))
    _compare(got, want)
    assert rel_l2(got_views.cpu().numpy(), want_views.cpu().numpy()) <= TOL
    # a second step adds its gradient to the existing p.grad
    sync = GradientSync(*leaves, buckets=5)
    again, _ = _step(s, leaves, cams, dev, sync)
    _compare(again, [2 * w for w in want])


def test_gradient_sync_one_rank_nccl_group():
    from dsl_splat_b200.sharding import GradientSync
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    s = _scene()
    want, _ = _step(s, _leaves(s, dev), [1, 3], dev)
    dist.init_process_group("nccl", store=dist.HashStore(), rank=0, world_size=1,
                            device_id=dev)
    try:
        leaves = _leaves(s, dev)
        got, _ = _step(s, leaves, [1, 3], dev,
                       GradientSync(*leaves, group=dist.group.WORLD, buckets=4))
    finally:
        dist.destroy_process_group()
    _compare(got, want)


def _free_port():
    sock = socket.socket()
    sock.bind(("127.0.0.1", 0))
    port = sock.getsockname()[1]
    sock.close()
    return port


def _rank(rank, world, port, outdir):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    from dsl_splat_b200 import sharding
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    sharding.init_process_group("nccl", timeout_s=60.0, device=dev)
    s = _scene()
    cams = sharding.local_cameras(s.viewmats.shape[0], rank, world)
    leaves = _leaves(s, dev)
    got, _ = _step(s, leaves, cams, dev,
                   sharding.GradientSync(*leaves, group=dist.group.WORLD, buckets=4))
    out = {"grads": [g.cpu() for g in got]}
    if rank == 0:
        want, _ = _step(s, _leaves(s, dev), list(range(s.viewmats.shape[0])), dev)
        out["want"] = [w.cpu() for w in want]
    torch.save(out, os.path.join(outdir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_gradient_sync_across_gpus(tmp_path):
    world = min(torch.cuda.device_count(), 4)
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank, args=(r, world, port, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
        assert p.exitcode == 0
    want = torch.load(os.path.join(tmp_path, "rank0.pt"))["want"]
    for r in range(world):
        _compare(torch.load(os.path.join(tmp_path, f"rank{r}.pt"))["grads"], want)
