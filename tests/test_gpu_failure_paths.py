"""Failure paths of the tensor-core kernels and of the bulk-copy ring passes,
exercised without faulting the GPU.

Every wait of the tensor-core kernel (ra_tc16.cuh) on an mbarrier is bounded;
when one expires the kernel records a timeout in the workspace's error word,
its roles stop (the epilogue warps agree on it before any named barrier),
it waits for the copies it issued, frees its tensor memory and returns, and
ra_kde_check reports RA_ERR_DEVICE_TIMEOUT.  The test hook RA_TEST_NO_MMA makes the kernels issue no
MMA at all and bound each wait to 4096 polls: the first wait for a GEMM then
expires with nothing asynchronous in flight.  Each test checks the status, then
runs the same problem normally on the same device and compares it with the
oracle, which also shows that the aborted launch freed its tensor memory (a
persistent CTA of the next launch could not allocate it otherwise).
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

K_TOL = 2e-6


def _problem(seed, sizes, dim, dev):
    rng = np.random.default_rng(seed)
    ptr = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    x = (rng.standard_normal((ptr[-1], dim)) / np.sqrt(dim)).astype(np.float32)
    y = (x + 0.1 * rng.standard_normal(x.shape)).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(dev).contiguous()
    return x, y, ptr, t(x), t(y), t(ptr)


def _forward(lib, xt, yt, pt, P, dim, sigma, hooks, need_grad, dev):
    from rapidalign_b200 import _lib
    d = _lib.RaKdeDesc()
    d.num_pairs, d.dim, d.layout = P, dim, _lib.RA_LAYOUT_RAGGED
    d.num_x, d.num_y = xt.shape[0], yt.shape[0]
    d.weights_x = d.weights_y = _lib.RA_WEIGHTS_UNIFORM
    d.center, d.need_grad, d.need_sigma_grad = 0, need_grad, 0
    d.shard_index, d.shard_count = 0, 1
    d.sigma, d.engine, d.test_hooks = sigma, _lib.RA_ENGINE_TENSOR, hooks
    inp = _lib.RaKdeInputs()
    inp.x, inp.y, inp.ptr_x, inp.ptr_y = xt.data_ptr(), yt.data_ptr(), pt.data_ptr(), pt.data_ptr()
    nbytes = lib.ra_kde_workspace_bytes(ctypes.byref(d))
    assert nbytes > 0
    ws = _lib.workspace(nbytes, dev)
    K = torch.zeros(3 * P, dtype=torch.float64, device=dev)
    stream = _lib.stream_handle(dev)
    rc = lib.ra_kde_forward(ctypes.byref(d), ctypes.byref(inp), K.data_ptr(), ws.data_ptr(),
                            ws.numel(), stream)
    assert rc == 0, _lib.status_string(rc)
    return K, lib.ra_kde_check(ws.data_ptr(), stream)


@pytest.mark.parametrize("dim,need_grad", [(32, 0), (32, 1), (128, 0), (128, 1)])
def test_expired_wait_is_reported_and_the_device_stays_usable(dim, need_grad, cuda_device):
    """Padded widths 32 and 128 of the same kernel (different TMEM and
    shared-memory footprints)."""
    from rapidalign_b200 import _lib
    lib = _lib.load()
    dev = cuda_device
    sizes = [300, 70, 129]
    x, y, ptr, xt, yt, pt = _problem(31 + dim, sizes, dim, dev)
    sigma = 1.0
    _, status = _forward(lib, xt, yt, pt, len(sizes), dim, sigma, _lib.RA_TEST_NO_MMA,
                         need_grad, dev)
    assert status == _lib.RA_ERR_DEVICE_TIMEOUT, _lib.status_string(status)
    # the same problem, normally, twice (a second launch needs every SM's TMEM)
    for _ in range(2):
        K, status = _forward(lib, xt, yt, pt, len(sizes), dim, sigma, 0, need_grad, dev)
        assert status == _lib.RA_OK, _lib.status_string(status)
        P = len(sizes)
        a = np.concatenate([np.full(n, 1.0 / n) for n in sizes])
        rs = O.raw_sums(x, y, a, a, ptr, ptr, sigma)
        got = K.cpu().numpy().reshape(3, P)
        for k in range(3):
            assert np.all(np.abs(got[k] - rs.K[:, k]) <= K_TOL * np.abs(rs.K[:, k])), k


def _forward_backward(lib, xt, yt, pt, P, dim, sigma, hooks_fwd, hooks_bwd, dev):
    """Forward then backward (coefficients of the MMD loss, 1, 1, -2) on one
    workspace; the status after each, the sums and the position gradients."""
    from rapidalign_b200 import _lib
    d = _lib.RaKdeDesc()
    d.num_pairs, d.dim, d.layout = P, dim, _lib.RA_LAYOUT_RAGGED
    d.num_x, d.num_y = xt.shape[0], yt.shape[0]
    d.weights_x = d.weights_y = _lib.RA_WEIGHTS_UNIFORM
    d.center, d.need_grad, d.need_sigma_grad, d.skip_weight_sums = 0, 1, 0, 1
    d.shard_index, d.shard_count = 0, 1
    d.sigma, d.engine, d.test_hooks = sigma, _lib.RA_ENGINE_TENSOR, hooks_fwd
    inp = _lib.RaKdeInputs()
    inp.x, inp.y, inp.ptr_x, inp.ptr_y = xt.data_ptr(), yt.data_ptr(), pt.data_ptr(), pt.data_ptr()
    ws = _lib.workspace(lib.ra_kde_workspace_bytes(ctypes.byref(d)), dev)
    K = torch.zeros(3 * P, dtype=torch.float64, device=dev)
    stream = _lib.stream_handle(dev)
    rc = lib.ra_kde_forward(ctypes.byref(d), ctypes.byref(inp), K.data_ptr(), ws.data_ptr(),
                            ws.numel(), stream)
    assert rc == 0, _lib.status_string(rc)
    status_fwd = lib.ra_kde_check(ws.data_ptr(), stream)
    coef = torch.cat([torch.ones(2 * P), torch.full((P,), -2.0)]).to(dev, torch.float64)
    gx, gy = torch.zeros_like(xt), torch.zeros_like(yt)
    g = _lib.RaKdeGrads()
    g.grad_x, g.grad_y = gx.data_ptr(), gy.data_ptr()
    d.test_hooks = hooks_bwd
    rc = lib.ra_kde_backward(ctypes.byref(d), ctypes.byref(inp), coef.data_ptr(), ctypes.byref(g),
                             ws.data_ptr(), ws.numel(), stream)
    assert rc == 0, _lib.status_string(rc)
    status_bwd = lib.ra_kde_check(ws.data_ptr(), stream)
    return K, status_fwd, status_bwd, gx, gy


@pytest.mark.parametrize("dim", [32, 128])
def test_ring_pass_expired_wait_is_reported(dim, cuda_device):
    """The O(N) passes that stream rows by bulk copies (equal weights, no
    mask): with RA_TEST_RING_IDLE their producers copy nothing and every wait
    is bounded to 4096 polls, so the consumers' first wait expires.  The
    forward's passes (sums, packing) report RA_ERR_DEVICE_TIMEOUT, and so does
    the backward's write pass after a normal forward; then normal calls on the
    same device match the oracle, K and gradients (a 1500-point side spans two
    chunks)."""
    from rapidalign_b200 import _lib
    from test_gpu_parity import assert_grad
    lib = _lib.load()
    dev = cuda_device
    sizes = [300, 70, 1500]
    P = len(sizes)
    x, y, ptr, xt, yt, pt = _problem(71 + dim, sizes, dim, dev)
    sigma = 1.0
    _, st_f, _, _, _ = _forward_backward(lib, xt, yt, pt, P, dim, sigma, _lib.RA_TEST_RING_IDLE,
                                         0, dev)
    assert st_f == _lib.RA_ERR_DEVICE_TIMEOUT, _lib.status_string(st_f)
    _, st_f, st_b, _, _ = _forward_backward(lib, xt, yt, pt, P, dim, sigma, 0,
                                            _lib.RA_TEST_RING_IDLE, dev)
    assert st_f == _lib.RA_OK, _lib.status_string(st_f)
    assert st_b == _lib.RA_ERR_DEVICE_TIMEOUT, _lib.status_string(st_b)
    r = O.pyg_kde_mmd_loss(x, y, ptr, ptr, sigma=sigma, center=False,
                           upstream=[np.ones(P), np.zeros(P), np.zeros(P), np.zeros(P)])
    for _ in range(2):
        K, st_f, st_b, gx, gy = _forward_backward(lib, xt, yt, pt, P, dim, sigma, 0, 0, dev)
        assert st_f == _lib.RA_OK and st_b == _lib.RA_OK, (st_f, st_b)
        got = K.cpu().numpy().reshape(3, P)
        for k, ref in enumerate((r.Kxx, r.Kyy, r.Kxy)):
            assert np.all(np.abs(got[k] - ref) <= K_TOL * np.abs(ref)), k
        assert_grad(gx.cpu().numpy(), r.grad_x, "grad_x")
        assert_grad(gy.cpu().numpy(), r.grad_y, "grad_y")
