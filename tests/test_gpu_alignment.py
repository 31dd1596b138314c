"""Caller buffers that are contiguous but not 16-byte aligned.

The wide-point passes (padded width >= 32) read the caller's coordinates and
write its position gradients as float4 when D % 4 == 0.  A contiguous tensor
can start at any float (a view at storage offset 1, or a raw pointer through
the C ABI), and a float4 access there would be a misaligned-address fault, so
the library checks the pointers on the host and takes the scalar passes for
any that are not 16-byte aligned.  These tests run both kinds of call on the
same data and compare them with each other and with the float64 oracle.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from test_gpu_parity import _np, assert_grad, assert_k

pytestmark = pytest.mark.gpu


def _offset_copy(a: np.ndarray, dev, grad=False) -> torch.Tensor:
    """A contiguous float32 CUDA tensor holding `a` that starts 4 bytes past
    a 16-byte boundary (a view at storage offset 1 of a fresh allocation)."""
    buf = torch.zeros(a.size + 1, dtype=torch.float32, device=dev)
    t = buf[1:].view(a.shape)
    t.copy_(torch.from_numpy(np.ascontiguousarray(a)))
    assert t.is_contiguous() and t.data_ptr() % 16 == 4
    if grad:
        t.requires_grad_(True)
    return t


def _batch(seed, sizes, d):
    rng = np.random.default_rng(seed)
    ptr = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    x = (rng.standard_normal((ptr[-1], d)) / np.sqrt(d)).astype(np.float32)
    y = (x + 0.1 * rng.standard_normal(x.shape)).astype(np.float32)
    return x, y, ptr


@pytest.mark.parametrize("d", [32, 64, 128, 256])
@pytest.mark.parametrize("center", [False, True])
def test_unaligned_points_match_aligned_and_oracle(d, center, cuda_device):
    """d = 32, 64, 128: tensor-core tiles; d = 256: the SIMT tiles.  Without
    centering and weights the backward also skips its side-totals pass."""
    import rapidalign_b200 as ra
    dev = cuda_device
    x, y, ptr = _batch(60 + d + int(center), [300, 65, 1, 129], d)
    pt = torch.from_numpy(ptr).to(dev)
    res = {}
    for kind in ("aligned", "offset"):
        if kind == "aligned":
            xt = torch.from_numpy(x).to(dev).requires_grad_(True)
            yt = torch.from_numpy(y).to(dev).requires_grad_(True)
            assert xt.data_ptr() % 16 == 0 and yt.data_ptr() % 16 == 0
        else:
            xt, yt = _offset_copy(x, dev, True), _offset_copy(y, dev, True)
        loss, kxx, kyy, kxy = ra.pyg_kde_mmd_loss(xt, yt, src_ptr=pt, tgt_ptr=pt, sigma=1.0,
                                                  center=center)
        loss.sum().backward()
        res[kind] = [_np(v) for v in (loss, kxx, kyy, kxy, xt.grad, yt.grad)]
    r = O.pyg_kde_mmd_loss(x, y, ptr, ptr, sigma=1.0, center=center,
                           upstream=[np.ones(4), np.zeros(4), np.zeros(4), np.zeros(4)])
    for kind, (loss, kxx, kyy, kxy, gx, gy) in res.items():
        assert_k(kxx, r.Kxx, f"Kxx {kind}")
        assert_k(kyy, r.Kyy, f"Kyy {kind}")
        assert_k(kxy, r.Kxy, f"Kxy {kind}")
        assert_grad(gx, r.grad_x, f"grad_x {kind}")
        assert_grad(gy, r.grad_y, f"grad_y {kind}")
    # the two call kinds take different O(N) kernels (aligned points: the
    # bulk-copy passes; offset points: scalar loads), which add the fp64 side
    # sums and the fp32 |x'|^2 of each point in different orders: a few
    # float32 roundings apart, far inside the oracle tolerance above
    for a, b in zip(res["aligned"], res["offset"]):
        scale = max(float(np.abs(a).max()), 1e-30)
        assert float(np.abs(a - b).max()) <= 4e-6 * scale


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("center", [0, 1])
def test_unaligned_gradient_buffers_through_the_c_abi(d, center, cuda_device):
    """ra_kde_backward writing into grad_x / grad_y that start 4 bytes past a
    16-byte boundary: the same gradients as into aligned buffers."""
    from rapidalign_b200 import _lib
    lib = _lib.load()
    dev = cuda_device
    x, y, ptr = _batch(70 + d + center, [200, 64, 130], d)
    xt, yt, pt = (torch.from_numpy(a).to(dev) for a in (x, y, ptr))
    P = len(ptr) - 1
    desc = _lib.RaKdeDesc()
    desc.num_pairs, desc.dim, desc.layout = P, d, _lib.RA_LAYOUT_RAGGED
    desc.num_x, desc.num_y = x.shape[0], y.shape[0]
    desc.weights_x = desc.weights_y = _lib.RA_WEIGHTS_UNIFORM
    desc.center, desc.need_grad, desc.need_sigma_grad = center, 1, 0
    desc.shard_index, desc.shard_count = 0, 1
    desc.sigma, desc.engine = 1.0, _lib.RA_ENGINE_AUTO
    inp = _lib.RaKdeInputs()
    inp.x, inp.y, inp.ptr_x, inp.ptr_y = xt.data_ptr(), yt.data_ptr(), pt.data_ptr(), pt.data_ptr()
    nbytes = lib.ra_kde_workspace_bytes(ctypes.byref(desc))
    assert nbytes > 0
    ws = _lib.workspace(nbytes, dev)
    K = torch.zeros(3 * P, dtype=torch.float64, device=dev)
    stream = _lib.stream_handle(dev)
    rc = lib.ra_kde_forward(ctypes.byref(desc), ctypes.byref(inp), K.data_ptr(), ws.data_ptr(),
                            ws.numel(), stream)
    assert rc == 0, _lib.status_string(rc)
    coef = torch.tensor([1.0] * P + [1.0] * P + [-2.0] * P, dtype=torch.float64, device=dev)
    out = {}
    for kind in ("aligned", "offset"):
        if kind == "aligned":
            gx, gy = torch.empty_like(xt), torch.empty_like(yt)
        else:
            gx, gy = _offset_copy(np.zeros_like(x), dev), _offset_copy(np.zeros_like(y), dev)
        grads = _lib.RaKdeGrads()
        grads.grad_x, grads.grad_y = gx.data_ptr(), gy.data_ptr()
        grads.grad_wx = grads.grad_wy = grads.grad_sigma = None
        rc = lib.ra_kde_backward(ctypes.byref(desc), ctypes.byref(inp), coef.data_ptr(),
                                 ctypes.byref(grads), ws.data_ptr(), ws.numel(), stream)
        assert rc == 0, _lib.status_string(rc)
        assert lib.ra_kde_check(ws.data_ptr(), stream) == 0
        out[kind] = (_np(gx), _np(gy))
    r = O.pyg_kde_mmd_loss(x, y, ptr, ptr, sigma=1.0, center=bool(center),
                           upstream=[np.ones(P), np.zeros(P), np.zeros(P), np.zeros(P)])
    for kind, (gx, gy) in out.items():
        assert_grad(gx, r.grad_x, f"grad_x {kind}")
        assert_grad(gy, r.grad_y, f"grad_y {kind}")
    for a, b in zip(out["aligned"], out["offset"]):
        assert float(np.abs(a - b).max()) <= 1e-6 * max(float(np.abs(a).max()), 1e-30)
