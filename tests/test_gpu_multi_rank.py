"""Multi-GPU paths on 2 GPUs of one box, one process per GPU over NCCL.

* split_pair_kde_mmd_loss (one pair split across the ranks by work items,
  one all-reduce of the packed partial sums) against the unsplit
  kde_mmd_loss (rapidalign/kde.py:39-109) on each rank: K, loss and every
  gradient;
* sharded_pyg_kde_mmd_loss and sharded_kde_mmd_loss_dense (graphs / clouds
  LPT-partitioned across the ranks, one all_gather) against the one-GPU
  pyg_kde_mmd_loss / kde_mmd_loss_dense: every graph's results on every rank
  and, summed over the ranks, the gradients.

The ranks run as spawned child processes with a short NCCL timeout and NVLS
off, and the parent bounds the wait for them.  Skipped with fewer than 2 GPUs.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

K_TOL = 2e-6
LOSS_TOL = 1e-5
GRAD_TOL = 1e-4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    import rapidalign_b200 as ra
    from rapidalign_b200 import shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    out = {}
    rng = np.random.default_rng(21)
    # ---- one pair split over the ranks -------------------------------------
    n, m = 20000, 19000
    x = rng.standard_normal((n, 3)).astype(np.float32)
    y = (rng.standard_normal((m, 3)) * 0.9 + 0.05).astype(np.float32)
    w = (rng.random(n) + 0.1).astype(np.float32)
    for tag, split in (("split", True), ("whole", False)):
        xt = torch.from_numpy(x).to(dev).requires_grad_(True)
        yt = torch.from_numpy(y).to(dev).requires_grad_(True)
        wt = torch.from_numpy(w).to(dev).requires_grad_(True)
        if split:
            res = shard.split_pair_kde_mmd_loss(xt, yt, wt, None, sigma=0.2, center=True)
        else:
            res = ra.kde_mmd_loss(xt, yt, wt, None, sigma=0.2, center=True)
        (res[0] + 0.3 * res[3]).backward()
        out[tag + "_K"] = np.array([float(v) for v in res])
        out[tag + "_gx"] = xt.grad.cpu().numpy()
        out[tag + "_gy"] = yt.grad.cpu().numpy()
        out[tag + "_gw"] = wt.grad.cpu().numpy()
    # ---- a ragged batch sharded by graphs ----------------------------------
    sizes_x = [300, 5, 1200, 77, 640, 64, 65, 900]
    sizes_y = [290, 9, 1100, 80, 700, 60, 70, 880]
    px = np.concatenate([[0], np.cumsum(sizes_x)])
    py = np.concatenate([[0], np.cumsum(sizes_y)])
    bx = rng.standard_normal((px[-1], 3)).astype(np.float32)
    by = rng.standard_normal((py[-1], 3)).astype(np.float32)
    for tag, sharded in (("rsh", True), ("rone", False)):
        xt = torch.from_numpy(bx).to(dev).requires_grad_(True)
        yt = torch.from_numpy(by).to(dev).requires_grad_(True)
        ptx, pty = torch.from_numpy(px).to(dev), torch.from_numpy(py).to(dev)
        if sharded:
            res = shard.sharded_pyg_kde_mmd_loss(xt, yt, ptx, pty, sigma=0.25)
        else:
            res = ra.pyg_kde_mmd_loss(xt, yt, src_ptr=ptx, tgt_ptr=pty, sigma=0.25)
        res[0].sum().backward()
        out[tag + "_res"] = torch.stack([r.detach().double() for r in res]).cpu().numpy()
        out[tag + "_gx"] = xt.grad.cpu().numpy()
    # ---- a dense batch sharded by clouds -----------------------------------
    B, N = 6, 700
    dx = rng.standard_normal((B, N, 3)).astype(np.float32)
    dy = (dx + 0.05 * rng.standard_normal((B, N, 3))).astype(np.float32)
    mx = np.arange(N)[None, :] < rng.integers(300, N + 1, B)[:, None]
    my = np.arange(N)[None, :] < rng.integers(300, N + 1, B)[:, None]
    for tag, sharded in (("dsh", True), ("done", False)):
        xt = torch.from_numpy(dx).to(dev).requires_grad_(True)
        yt = torch.from_numpy(dy).to(dev)
        mxt, myt = torch.from_numpy(mx).to(dev), torch.from_numpy(my).to(dev)
        if sharded:
            res = shard.sharded_kde_mmd_loss_dense(xt, yt, mxt, myt, sigma=0.25)
        else:
            res = ra.kde_mmd_loss_dense(xt, yt, mxt, myt, sigma=0.25)
        res[0].sum().backward()
        out[tag + "_res"] = torch.stack([r.detach().double() for r in res]).cpu().numpy()
        out[tag + "_gx"] = xt.grad.cpu().numpy()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **out)
    dist.barrier()
    dist.destroy_process_group()


def _rel(a, b):
    return float(np.max(np.abs(a - b) / np.abs(b)))


def _gerr(a, b):
    return float(np.max(np.abs(a - b)) / np.max(np.abs(b)))


def test_two_ranks_match_one_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    world = 2
    ctx = mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                             join=False, start_method="spawn")
    for _ in range(30):  # at most 300 s
        if ctx.join(timeout=10):
            break
    else:
        for p in ctx.processes:
            if p.is_alive():
                p.kill()
        pytest.fail("the ranks did not finish in 300 s")
    zs = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    for z in zs:
        # split pair == unsplit pair, on every rank
        K, ref = z["split_K"], z["whole_K"]
        assert abs(K[0] - ref[0]) <= LOSS_TOL * abs(ref[0])
        assert np.all(np.abs(K[1:] - ref[1:]) <= K_TOL * np.abs(ref[1:]))
        for g in ("gx", "gy", "gw"):
            assert _gerr(z["split_" + g], z["whole_" + g]) <= GRAD_TOL, g
        # every graph's results on every rank
        for tag in ("r", "d"):
            got, ref = z[tag + "sh_res"], z[tag + "one_res"]
            assert np.all(np.abs(got - ref) <= K_TOL * np.abs(ref) + 1e-12), tag
    # each rank's backward covers its own graphs: the sum is the whole gradient
    for tag in ("r", "d"):
        total = sum(z[tag + "sh_gx"] for z in zs)
        assert _gerr(total, zs[0][tag + "one_gx"]) <= GRAD_TOL, tag
