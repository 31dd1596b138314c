"""The no-allocation ragged forward, ra_kde_mmd_forward_segmented_noalloc.

It exists for callers that cannot allocate device memory (a host that keeps
all device memory in its own pool, a loop that must not allocate once it
runs): it takes only inputs and outputs and works in a fixed scratch array
inside the library.  Checked here through the C ABI against the ordinary
entry point (caller-supplied workspace) on two calls in a row, so that the
second call also shows that the contents the first call left in the shared
scratch do not leak into its results.  Collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

K_TOL = 2e-6  # same relative tolerance on K as the other parity tests


def _problem(seed, sizes_x, sizes_y, dev, dim=3):
    rng = np.random.default_rng(seed)
    ptr_x = np.concatenate([[0], np.cumsum(sizes_x)]).astype(np.int64)
    ptr_y = np.concatenate([[0], np.cumsum(sizes_y)]).astype(np.int64)
    x = rng.standard_normal((ptr_x[-1], dim)).astype(np.float32)
    y = rng.standard_normal((ptr_y[-1], dim)).astype(np.float32)
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
    # two different problems back to back: the second must not see the first
    problems = [
        (_problem(1, [130, 7, 64, 900], [120, 9, 70, 880], dev), 4, 0.25),
        (_problem(2, [33, 1, 500], [40, 2, 510], dev, dim=2), 3, 0.4),
    ]
    for args, P, sigma in problems:
        ref = _with_workspace(lib, args, P, sigma, dev)
        got = _no_alloc(lib, args, P, sigma, dev)
        torch.cuda.synchronize(dev)
        ref_np = ref.cpu().numpy()
        got_np = got.cpu().numpy()
        assert np.all(np.isfinite(got_np))
        assert np.all(np.abs(got_np - ref_np) <= K_TOL * np.abs(ref_np))


def test_no_alloc_rejects_problems_beyond_its_scratch(cuda_device):
    from rapidalign_b200 import _lib
    lib = _lib.load()
    P, NX, NY, D = 4096, 4_000_000, 4_000_000, 3  # workspace far above 64 MiB
    assert lib.ra_kde_mmd_forward_segmented_workspace_bytes(P, NX, NY, D) > (64 << 20)
    rc = lib.ra_kde_mmd_forward_segmented_noalloc(None, None, None, None, None, None, P, NX, NY,
                                                  D, 0.25, None, None, None, None)
    assert rc == _lib.RA_ERR_SCRATCH_LIMIT
    assert "64 MiB" in _lib.status_string(rc)
