"""Parity on the benchmark workloads themselves, at their full sizes.

The inputs are the exact ones ``bench.py`` times (its seeded generators), run
through the public API, forward and backward, and compared with the float64
oracle:

* ragged PyG batch: 4096 graphs of 32-2048 points, D=3, sigma 0.25, centred
  (``pyg_kde_mmd_loss`` with batch vectors; rapidalign/kde.py:302-428);
* dense padded batch: 64 clouds of 1024 points, valid 512-1024, D=3, sigma
  0.25, centred (``kde_mmd_loss_dense``; kde.py:211-299);
* graph embeddings: 1024 graphs of 64-512 nodes, D=128, sigma 1.0, uncentred
  (``pyg_kde_mmd_loss`` on the tensor-core path);
* one pair of 262144 points per cloud, D=3, sigma 0.2, centred
  (``kde_mmd_loss``; kde.py:39-109), against values the oracle computed once
  over the whole pair (``tests/golden/oracle/make_huge_pair_fixture.py``): K, the
  loss, and the gradients of 256 seeded rows of each cloud.

Bars (the target's own): losses within 1e-5 relative with no floor, K within
2e-6 relative, gradients within 1e-4 of the largest gradient component of the
tensor.  The embeddings' losses use the tensor-core path's stated bound
|dL| <= 1e-5 |L| + 1e-6 (Kxx + Kyy) (tests/test_gpu_tensor_core.py) and are
also checked at the plain 1e-5 relative bar, which holds on this data.
"""
import os

import numpy as np
import pytest
import torch

import bench
from conftest import GOLDEN_DIR
from oracle import oracle as O

pytestmark = pytest.mark.gpu

K_TOL = 2e-6
LOSS_TOL = 1e-5
GRAD_TOL = 1e-4


def _np(t):
    return t.detach().double().cpu().numpy()


def _rel(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref) / np.abs(ref)))


def _grad_err(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref))) / float(np.max(np.abs(ref)))


def _check(outs, ref, gx, gy, name, loss_tol=LOSS_TOL):
    errs = {
        "loss": _rel(_np(outs[0]), ref.loss),
        "Kxx": _rel(_np(outs[1]), ref.Kxx),
        "Kyy": _rel(_np(outs[2]), ref.Kyy),
        "Kxy": _rel(_np(outs[3]), ref.Kxy),
        "grad_x": _grad_err(_np(gx), ref.grad_x),
        "grad_y": _grad_err(_np(gy), ref.grad_y),
    }
    print(name, {k: f"{v:.2e}" for k, v in errs.items()})
    assert errs["loss"] <= loss_tol, (name, errs)
    for k in ("Kxx", "Kyy", "Kxy"):
        assert errs[k] <= K_TOL, (name, errs)
    assert errs["grad_x"] <= GRAD_TOL and errs["grad_y"] <= GRAD_TOL, (name, errs)
    return errs


def test_ragged_4096_graphs(cuda_device):
    import rapidalign_b200 as ra
    dev = cuda_device
    x, y, bx, by, nx, ny = bench.ragged_batch(range(bench.GRAPHS_PER_GPU))
    xt = torch.from_numpy(x).to(dev).requires_grad_(True)
    yt = torch.from_numpy(y).to(dev).requires_grad_(True)
    outs = ra.pyg_kde_mmd_loss(xt, yt, src_batch=torch.from_numpy(bx).to(dev),
                               tgt_batch=torch.from_numpy(by).to(dev), sigma=bench.SIGMA,
                               center=True)
    outs[0].sum().backward()
    P = len(nx)
    ptr_x = np.concatenate([[0], np.cumsum(nx)])
    ptr_y = np.concatenate([[0], np.cumsum(ny)])
    ref = O.pyg_kde_mmd_loss(x, y, ptr_x, ptr_y, sigma=bench.SIGMA, center=True,
                             upstream=[np.ones(P), np.zeros(P), np.zeros(P), np.zeros(P)])
    _check(outs, ref, xt.grad, yt.grad, "ragged 4096")


def test_dense_64_clouds_of_1024(cuda_device):
    import rapidalign_b200 as ra
    dev = cuda_device
    x, y, lx, ly = bench.dense_data(0)
    nmax = x.shape[1]
    mx = np.arange(nmax)[None, :] < lx[:, None]
    my = np.arange(nmax)[None, :] < ly[:, None]
    xt = torch.from_numpy(x).to(dev).requires_grad_(True)
    yt = torch.from_numpy(y).to(dev).requires_grad_(True)
    outs = ra.kde_mmd_loss_dense(xt, yt, torch.from_numpy(mx).to(dev),
                                 torch.from_numpy(my).to(dev), sigma=bench.SIGMA, center=True)
    outs[0].sum().backward()
    B = x.shape[0]
    ref = O.kde_mmd_loss_dense(x, y, mx, my, sigma=bench.SIGMA, center=True,
                               upstream=[np.ones(B), np.zeros(B), np.zeros(B), np.zeros(B)])
    _check(outs, ref, xt.grad, yt.grad, "dense 64x1024")


def test_embeddings_1024_graphs_d128(cuda_device):
    import rapidalign_b200 as ra
    dev = cuda_device
    xs, ys = zip(*(bench.embed_graph(g) for g in range(1024)))
    n = np.array([a.shape[0] for a in xs])
    x, y = np.concatenate(xs), np.concatenate(ys)
    ptr = np.concatenate([[0], np.cumsum(n)])
    xt = torch.from_numpy(x).to(dev).requires_grad_(True)
    yt = torch.from_numpy(y).to(dev).requires_grad_(True)
    pt = torch.from_numpy(ptr).to(dev)
    outs = ra.pyg_kde_mmd_loss(xt, yt, src_ptr=pt, tgt_ptr=pt, sigma=1.0, center=False)
    outs[0].sum().backward()
    P = len(n)
    ref = O.pyg_kde_mmd_loss(x, y, ptr, ptr, sigma=1.0, center=False,
                             upstream=[np.ones(P), np.zeros(P), np.zeros(P), np.zeros(P)])
    errs = _check(outs, ref, xt.grad, yt.grad, "embeddings 1024 x D128")
    # the tensor-core path's stated loss bound, checked per graph as well
    bound = LOSS_TOL * np.abs(ref.loss) + 1e-6 * (np.abs(ref.Kxx) + np.abs(ref.Kyy))
    assert np.all(np.abs(_np(outs[0]) - ref.loss) <= bound), errs


def test_huge_pair_262144(cuda_device):
    import rapidalign_b200 as ra
    path = os.path.join(GOLDEN_DIR, "oracle", "huge_pair_262144.npz")
    with np.load(path) as z:
        fix = {k: z[k] for k in z.files}
    dev = cuda_device
    src, tgt = bench.huge_pair_data(int(fix["n"]))
    xt = torch.from_numpy(src).to(dev).requires_grad_(True)
    yt = torch.from_numpy(tgt).to(dev).requires_grad_(True)
    loss, Kxx, Kyy, Kxy = ra.kde_mmd_loss(xt, yt, sigma=float(fix["sigma"]), center=True)
    loss.backward()
    errs = {
        "loss": _rel(loss.item(), fix["loss"]),
        "Kxx": _rel(Kxx.item(), fix["Kxx"]),
        "Kyy": _rel(Kyy.item(), fix["Kyy"]),
        "Kxy": _rel(Kxy.item(), fix["Kxy"]),
    }
    rows = fix["rows"]
    gx, gy = _np(xt.grad)[rows], _np(yt.grad)[rows]
    # judged against the largest component among the checked rows (a stricter
    # scale than the whole tensor's largest component, also stored)
    errs["grad_x"] = _grad_err(gx, fix["grad_x_rows"])
    errs["grad_y"] = _grad_err(gy, fix["grad_y_rows"])
    print("huge pair", {k: f"{v:.2e}" for k, v in errs.items()})
    assert errs["loss"] <= LOSS_TOL, errs
    for k in ("Kxx", "Kyy", "Kxy"):
        assert errs[k] <= K_TOL, errs
    assert errs["grad_x"] <= GRAD_TOL and errs["grad_y"] <= GRAD_TOL, errs
