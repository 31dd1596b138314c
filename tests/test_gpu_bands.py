"""kde_mmd_loss_bands: several bandwidths of one pair in one call (per-pair
bandwidths in the C ABI, ra_kde_inputs.sigma_pairs), against the float64
oracle band by band and against the single-band entry point."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from test_gpu_parity import _cuda, _np, assert_grad, assert_k, assert_loss

pytestmark = pytest.mark.gpu


def _clouds(rng, n, m, d):
    x = rng.standard_normal((n, d)).astype(np.float32)
    y = (1.1 * rng.standard_normal((m, d)) + 0.05).astype(np.float32)
    return x, y


@pytest.mark.parametrize("d,n,m,weighted", [(2, 60, 45, True), (3, 300, 280, False),
                                            (8, 70, 90, True)])
def test_bands_match_oracle(d, n, m, weighted, cuda_device):
    import rapidalign_b200 as ra
    rng = np.random.default_rng(60 + d)
    x, y = _clouds(rng, n, m, d)
    wx = rng.uniform(0.2, 1.0, n).astype(np.float32) if weighted else None
    wy = rng.uniform(0.2, 1.0, m).astype(np.float32) if weighted else None
    sig = np.array([0.3, 0.6, 1.2])
    dev = cuda_device
    xt, yt = _cuda(x, dev, True), _cuda(y, dev, True)
    wxt = _cuda(wx, dev, True) if weighted else None
    wyt = _cuda(wy, dev, True) if weighted else None
    st = torch.tensor(sig, dtype=torch.float64, device=dev, requires_grad=True)
    loss, Kxx, Kyy, Kxy = ra.kde_mmd_loss_bands(xt, yt, wxt, wyt, sigmas=st, center=True)
    assert loss.shape == (3,)
    up = rng.uniform(0.5, 1.5, 3)
    (loss.double() * torch.as_tensor(up, device=dev)).sum().backward()
    gx = np.zeros_like(x, dtype=np.float64)
    gy = np.zeros_like(y, dtype=np.float64)
    gwx = np.zeros(n) if weighted else None
    gwy = np.zeros(m) if weighted else None
    for b, s in enumerate(sig):
        r = O.kde_mmd_loss(x, y, wx, wy, sigma=s, center=True,
                           upstream=[up[b], 0.0, 0.0, 0.0])
        assert_k(_np(Kxx)[b], r.Kxx, "Kxx")
        assert_k(_np(Kyy)[b], r.Kyy, "Kyy")
        assert_k(_np(Kxy)[b], r.Kxy, "Kxy")
        assert_loss(_np(loss)[b], r.loss, r.Kxx, r.Kyy, "loss")
        assert abs(float(st.grad[b]) - r.grad_sigma) <= 1e-4 * abs(r.grad_sigma), b
        gx += r.grad_x
        gy += r.grad_y
        if weighted:
            gwx += r.grad_wx
            gwy += r.grad_wy
    assert_grad(_np(xt.grad), gx, "grad_x")
    assert_grad(_np(yt.grad), gy, "grad_y")
    if weighted:
        assert_grad(_np(wxt.grad), gwx, "grad_wx")
        assert_grad(_np(wyt.grad), gwy, "grad_wy")


def test_bands_equal_single_band_calls(cuda_device):
    """One call over S bandwidths returns what S single-band calls return."""
    import rapidalign_b200 as ra
    rng = np.random.default_rng(70)
    x, y = _clouds(rng, 500, 450, 3)
    dev = cuda_device
    xt, yt = _cuda(x, dev), _cuda(y, dev)
    sig = [0.1, 0.25, 0.7, 2.0]
    multi = ra.kde_mmd_loss_bands(xt, yt, sigmas=sig, center=False)
    for b, s in enumerate(sig):
        single = ra.kde_mmd_loss(xt, yt, sigma=s, center=False)
        for a, c in zip(multi, single):
            assert abs(float(a[b]) - float(c)) <= 1e-12 * abs(float(c)) + 1e-30


def test_bands_reject_bad_sigmas(cuda_device):
    import rapidalign_b200 as ra
    x = torch.randn(10, 3, device=cuda_device)
    with pytest.raises(ValueError, match="sigma must be positive"):
        ra.kde_mmd_loss_bands(x, x, sigmas=[0.2, -0.1])
    with pytest.raises(ValueError, match="1-D"):
        ra.kde_mmd_loss_bands(x, x, sigmas=[])


def test_per_pair_sigma_checked_on_device(cuda_device):
    """A C caller's non-positive per-pair bandwidth comes back as
    RA_ERR_SIGMA from the device check (here through the Python plumbing)."""
    from rapidalign_b200 import _lib
    from rapidalign_b200._core import Spec, forward_sums
    dev = cuda_device
    x = torch.randn(20, 3, device=dev)
    spec = Spec(layout=_lib.RA_LAYOUT_RAGGED, num_pairs=2, dim=3, num_x=20, num_y=20,
                center=False, sigma=1.0, ptr_x=torch.tensor([0, 10, 20], device=dev),
                ptr_y=torch.tensor([0, 10, 20], device=dev), check_errors=True,
                sigma_pairs=torch.tensor([0.5, -1.0], dtype=torch.float64, device=dev))
    with pytest.raises(ValueError, match="sigma must be positive"):
        forward_sums(x, x, None, None, None, spec, False)


def test_pyg_batch_adapter(cuda_device):
    """pyg_batch_kde_mmd_loss on batch-like objects: with ptr (no host sync)
    and with batch vectors only, equal to pyg_kde_mmd_loss."""
    from types import SimpleNamespace
    import rapidalign_b200 as ra
    from test_gpu_parity import _ragged
    rng = np.random.default_rng(71)
    x, y, ptr_x, ptr_y = _ragged(rng, [40, 7, 90], [35, 9, 88], 3)
    dev = cuda_device
    bx = np.repeat(np.arange(3), np.diff(ptr_x))
    by = np.repeat(np.arange(3), np.diff(ptr_y))
    wx = rng.uniform(0.2, 1.0, x.shape[0]).astype(np.float32)
    wy = rng.uniform(0.2, 1.0, y.shape[0]).astype(np.float32)
    src = SimpleNamespace(pos=_cuda(x, dev), batch=_cuda(bx, dev), ptr=_cuda(ptr_x, dev),
                          w=_cuda(wx, dev))
    tgt = SimpleNamespace(pos=_cuda(y, dev), batch=_cuda(by, dev), ptr=_cuda(ptr_y, dev),
                          w=_cuda(wy, dev))
    ref = ra.pyg_kde_mmd_loss(src.pos, tgt.pos, src_ptr=src.ptr, tgt_ptr=tgt.ptr, src_w=src.w,
                              tgt_w=tgt.w, sigma=0.3)
    a = ra.pyg_batch_kde_mmd_loss(src, tgt, weight="w", sigma=0.3)
    del src.ptr, tgt.ptr
    b = ra.pyg_batch_kde_mmd_loss(src, tgt, weight="w", sigma=0.3)
    for r, u, v in zip(ref, a, b):
        assert torch.equal(r, u) and torch.equal(r, v)
    with pytest.raises(ValueError, match="no attribute 'feat'"):
        ra.pyg_batch_kde_mmd_loss(src, tgt, weight="feat")
