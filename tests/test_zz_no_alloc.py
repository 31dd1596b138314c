"""The no-allocation ragged forward, ra_kde_mmd_forward_segmented_noalloc.

It exists for callers that cannot allocate device memory (a host that keeps
all device memory in its own pool, a loop that must not allocate once it
runs): it takes only inputs and outputs and works in a fixed scratch array
inside the library.  Checked here through the C ABI against the ordinary
entry point (caller-supplied workspace) on calls in a row, so that each later
call also shows that the contents an earlier call left in the shared scratch
do not leak into its results.  Both entry points run the same kernels with
the same fixed-order reductions, so their K values must be bitwise equal.
Collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _problem(seed, sizes_x, sizes_y, dev, dim=3):
    rng = np.random.default_rng(seed)
    ptr_x = np.concatenate([[0], np.cumsum(sizes_x)]).astype(np.int64)
    ptr_y = np.concatenate([[0], np.cumsum(sizes_y)]).astype(np.int64)
    x = (rng.standard_normal((ptr_x[-1], dim)) / np.sqrt(max(dim / 3, 1))).astype(np.float32)
    y = (rng.standard_normal((ptr_y[-1], dim)) / np.sqrt(max(dim / 3, 1))).astype(np.float32)
    wx = rng.random(ptr_x[-1]).astype(np.float32) + 0.1
    wy = rng.random(ptr_y[-1]).astype(np.float32) + 0.1
    t = lambda a: torch.from_numpy(a).to(dev).contiguous()
    return t(x), t(y), t(wx), t(wy), t(ptr_x), t(ptr_y)


def _with_workspace(lib, args, P, sigma, dev):
    from rapidalign_b200 import _lib
    x, y, wx, wy, px, py = args
    NX, D = x.shape
    NY = y.shape[0]
    K = torch.full((3, P), float("nan"), dtype=torch.float64, device=dev)
    ws = _lib.workspace(lib.ra_kde_mmd_forward_segmented_workspace_bytes(P, NX, NY, D), dev)
    rc = lib.ra_kde_mmd_forward_segmented(
        x.data_ptr(), y.data_ptr(), wx.data_ptr(), wy.data_ptr(), px.data_ptr(), py.data_ptr(),
        P, NX, NY, D, sigma, K[0].data_ptr(), K[1].data_ptr(), K[2].data_ptr(), ws.data_ptr(),
        ws.numel(), _lib.stream_handle(dev))
    assert rc == 0, _lib.status_string(rc)
    return K


def _no_alloc(lib, args, P, sigma, dev):
    from rapidalign_b200 import _lib
    x, y, wx, wy, px, py = args
    NX, D = x.shape
    NY = y.shape[0]
    K = torch.full((3, P), float("nan"), dtype=torch.float64, device=dev)
    rc = lib.ra_kde_mmd_forward_segmented_noalloc(
        x.data_ptr(), y.data_ptr(), wx.data_ptr(), wy.data_ptr(), px.data_ptr(), py.data_ptr(),
        P, NX, NY, D, sigma, K[0].data_ptr(), K[1].data_ptr(), K[2].data_ptr(),
        _lib.stream_handle(dev))
    assert rc == 0, _lib.status_string(rc)
    return K


def test_no_alloc_forward_matches_workspace_forward(cuda_device):
    from rapidalign_b200 import _lib
    lib = _lib.load()
    dev = cuda_device
    # different problems back to back: none may see what an earlier one left.
    # D = 3 and 2 run the point-cloud tile kernel; D = 32 the tensor-core
    # kernel with its packed-coordinate layout, also in the shared scratch.
    problems = [
        (_problem(1, [130, 7, 64, 900], [120, 9, 70, 880], dev), 4, 0.25),
        (_problem(2, [33, 1, 500], [40, 2, 510], dev, dim=2), 3, 0.4),
        (_problem(3, [300, 5, 129], [270, 0, 140], dev, dim=32), 3, 1.0),
        (_problem(1, [130, 7, 64, 900], [120, 9, 70, 880], dev), 4, 0.25),
    ]
    for args, P, sigma in problems:
        ref = _with_workspace(lib, args, P, sigma, dev)
        got = _no_alloc(lib, args, P, sigma, dev)
        assert lib.ra_kde_check_noalloc(_lib.stream_handle(dev)) == _lib.RA_OK
        ref_np = ref.cpu().numpy()
        got_np = got.cpu().numpy()
        assert np.all(np.isfinite(got_np))
        assert np.array_equal(got_np, ref_np)


def test_no_alloc_reports_device_detected_errors(cuda_device):
    """A ptr whose last offset is not the number of points is caught on the
    device and read back through ra_kde_check_noalloc; the next good call on
    the same scratch reports no error."""
    from rapidalign_b200 import _lib
    lib = _lib.load()
    dev = cuda_device
    x, y, wx, wy, px, py = _problem(5, [100, 50], [90, 60], dev)
    bad = px.clone()
    bad[-1] -= 1
    _no_alloc(lib, (x, y, wx, wy, bad, py), 2, 0.3, dev)
    assert lib.ra_kde_check_noalloc(_lib.stream_handle(dev)) == _lib.RA_ERR_PTR_END
    got = _no_alloc(lib, (x, y, wx, wy, px, py), 2, 0.3, dev)
    assert lib.ra_kde_check_noalloc(_lib.stream_handle(dev)) == _lib.RA_OK
    ref = _with_workspace(lib, (x, y, wx, wy, px, py), 2, 0.3, dev)
    assert np.array_equal(got.cpu().numpy(), ref.cpu().numpy())


def test_no_alloc_rejects_problems_beyond_its_scratch(cuda_device):
    from rapidalign_b200 import _lib
    lib = _lib.load()
    P, NX, NY, D = 4096, 4_000_000, 4_000_000, 3  # workspace far above 64 MiB
    assert lib.ra_kde_mmd_forward_segmented_workspace_bytes(P, NX, NY, D) > (64 << 20)
    rc = lib.ra_kde_mmd_forward_segmented_noalloc(None, None, None, None, None, None, P, NX, NY,
                                                  D, 0.25, None, None, None, None)
    assert rc == _lib.RA_ERR_SCRATCH_LIMIT
    assert "64 MiB" in _lib.status_string(rc)
