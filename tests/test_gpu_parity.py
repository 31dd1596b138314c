"""Parity of the CUDA path with the reference (golden vectors) and the oracle.

Tolerances (float32 kernels with float64 sums vs float64 reference):
  * K values:    relative 2e-6;
  * losses:      relative 1e-5, where "relative" is against
                 max(|L|, 1e-4 * (Kxx + Kyy)) so that near-zero MMD values
                 (identical clouds) are judged against the size of the sums
                 that cancel in them;
  * gradients:   max |g - g_ref| / max |g_ref| <= 1e-4 per tensor.
"""
import numpy as np
import pytest
import torch

from conftest import golden_cases, load_golden
from oracle import oracle as O

pytestmark = pytest.mark.gpu

K_TOL = 2e-6
LOSS_TOL = 1e-5
GRAD_TOL = 1e-4


def _np(t):
    return t.detach().double().cpu().numpy()


def assert_k(got, ref, name=""):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    err = np.abs(got - ref) / np.maximum(np.abs(ref), 1e-300)
    assert np.all((err <= K_TOL) | (np.abs(ref) < 1e-30)), (name, float(err.max()))


def assert_loss(got, ref, kxx, kyy, name=""):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    scale = np.maximum(np.abs(ref), 1e-4 * (np.abs(kxx) + np.abs(kyy)))
    scale = np.maximum(scale, 1e-300)
    err = np.abs(got - ref) / scale
    assert np.all(err <= LOSS_TOL), (name, float(err.max()))


def assert_grad(got, ref, name=""):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    scale = max(float(np.max(np.abs(ref))) if ref.size else 0.0, 1e-300)
    err = float(np.max(np.abs(got - ref))) / scale if ref.size else 0.0
    assert err <= GRAD_TOL, (name, err)


def _cuda(a, dev, grad=False, dtype=torch.float32):
    t = torch.as_tensor(np.asarray(a)).to(dev)
    if t.is_floating_point():
        t = t.to(dtype)
    if grad:
        t.requires_grad_(True)
    return t


@pytest.mark.parametrize("name", golden_cases("single") + golden_cases("pyg") +
                         golden_cases("dense"))
def test_public_api_matches_golden(name, cuda_device):
    import rapidalign_b200 as ra
    z = load_golden(name)
    dev = cuda_device
    x = _cuda(z["x"], dev, True)
    y = _cuda(z["y"], dev, True)
    xw = _cuda(z["x_w"], dev, True) if "x_w" in z else None
    yw = _cuda(z["y_w"], dev, True) if "y_w" in z else None
    kw = dict(center=bool(z["center"]), cosine=bool(z["cosine"]))
    sig_t = None
    if name.startswith("single"):
        if bool(z["sigma_grad"]):
            sig_t = torch.tensor(float(z["sigma"]), dtype=torch.float32, device=dev,
                                 requires_grad=True)
        outs = ra.kde_mmd_loss(x, y, xw, yw, sigma=sig_t if sig_t is not None
                               else float(z["sigma"]), **kw)
    elif name.startswith("pyg"):
        if bool(z["use_batch"]):
            bx = torch.repeat_interleave(torch.arange(len(z["ptr_x"]) - 1),
                                         torch.as_tensor(np.diff(z["ptr_x"]))).to(dev)
            by = torch.repeat_interleave(torch.arange(len(z["ptr_y"]) - 1),
                                         torch.as_tensor(np.diff(z["ptr_y"]))).to(dev)
            outs = ra.pyg_kde_mmd_loss(x, y, src_batch=bx, tgt_batch=by, src_w=xw, tgt_w=yw,
                                       sigma=float(z["sigma"]), **kw)
        else:
            outs = ra.pyg_kde_mmd_loss(x, y, src_ptr=_cuda(z["ptr_x"], dev),
                                       tgt_ptr=_cuda(z["ptr_y"], dev), src_w=xw, tgt_w=yw,
                                       sigma=float(z["sigma"]), **kw)
    else:
        outs = ra.kde_mmd_loss_dense(x, y, _cuda(z["mask_x"], dev), _cuda(z["mask_y"], dev),
                                     x_w=xw, y_w=yw, sigma=float(z["sigma"]), **kw)
    loss, Kxx, Kyy, Kxy = outs
    assert_k(_np(Kxx), z["Kxx"], "Kxx")
    assert_k(_np(Kyy), z["Kyy"], "Kyy")
    assert_k(_np(Kxy), z["Kxy"], "Kxy")
    assert_loss(_np(loss), z["loss"], z["Kxx"], z["Kyy"], "loss")
    up = z["upstream"]
    total = sum((torch.as_tensor(u, device=dev, dtype=torch.float64) * o.double()).sum()
                for u, o in zip(up, outs))
    total.backward()
    assert_grad(_np(x.grad), z["grad_x"], "grad_x")
    assert_grad(_np(y.grad), z["grad_y"], "grad_y")
    if "grad_wx" in z:
        assert_grad(_np(xw.grad), z["grad_wx"], "grad_wx")
        assert_grad(_np(yw.grad), z["grad_wy"], "grad_wy")
    if "grad_sigma" in z:
        g = float(sig_t.grad)
        ref = float(z["grad_sigma"])
        assert abs(g - ref) <= GRAD_TOL * max(abs(ref), 1e-12), (g, ref)


@pytest.mark.parametrize("name", golden_cases("segmented"))
def test_segmented_loss_matches_golden(name, cuda_device):
    import rapidalign_b200 as ra
    z = load_golden(name)
    dev = cuda_device
    x = _cuda(z["x"], dev, True)
    y = _cuda(z["y"], dev, True)
    wx = _cuda(z["w_x"], dev, True, dtype=torch.float64)
    wy = _cuda(z["w_y"], dev, True, dtype=torch.float64)
    sig = torch.tensor(float(z["sigma"]), dtype=torch.float64, device=dev, requires_grad=True)
    losses = ra.segmented_kde_loss(x, y, wx, wy, _cuda(z["ptr_x"], dev), _cuda(z["ptr_y"], dev),
                                   sig)
    assert losses.dtype == torch.float64
    kxx = np.asarray(z["raw_Kxx"])
    kyy = np.asarray(z["raw_Kyy"])
    assert_loss(_np(losses), z["loss"], kxx, kyy, "loss")
    (losses * torch.as_tensor(z["upstream"], device=dev)).sum().backward()
    assert_grad(_np(x.grad), z["grad_x"], "grad_x")
    assert_grad(_np(y.grad), z["grad_y"], "grad_y")
    assert_grad(_np(wx.grad), z["grad_wx"], "grad_wx")
    assert_grad(_np(wy.grad), z["grad_wy"], "grad_wy")
    assert abs(float(sig.grad) - float(z["grad_sigma"])) <= GRAD_TOL * abs(float(z["grad_sigma"]))


def _ragged(rng, sizes_x, sizes_y, d, noise=0.05):
    ptr_x = np.concatenate([[0], np.cumsum(sizes_x)]).astype(np.int64)
    ptr_y = np.concatenate([[0], np.cumsum(sizes_y)]).astype(np.int64)
    x = rng.standard_normal((ptr_x[-1], d)).astype(np.float32)
    y = rng.standard_normal((ptr_y[-1], d)).astype(np.float32)
    for p in range(len(sizes_x)):
        k = min(sizes_x[p], sizes_y[p])
        y[ptr_y[p]:ptr_y[p] + k] = x[ptr_x[p]:ptr_x[p] + k] + noise * rng.standard_normal(
            (k, d)).astype(np.float32)
    return x, y, ptr_x, ptr_y


@pytest.mark.parametrize("d", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("sizes", [
    ([1, 2, 63, 64, 65, 129, 0, 300], [3, 1, 64, 70, 60, 128, 5, 0]),
    ([700, 33], [650, 40]),
])
def test_legacy_segmented_ops_match_oracle(d, sizes, cuda_device):
    """_cuda.kde_mmd_forward_segmented / kde_mmd_backward_segmented (raw,
    possibly negative weights, empty segments, sizes around the 64 tile)."""
    from rapidalign_b200 import _cuda as C
    rng = np.random.default_rng(100 + d)
    x, y, ptr_x, ptr_y = _ragged(rng, *sizes, d)
    wx = rng.standard_normal(x.shape[0]).astype(np.float32)
    wy = rng.standard_normal(y.shape[0]).astype(np.float32)
    sigma = 0.3
    dev = cuda_device
    args = [_cuda(v, dev) for v in (x, y, wx, wy)] + [_cuda(ptr_x, dev), _cuda(ptr_y, dev)]
    Kxx, Kyy, Kxy = C.kde_mmd_forward_segmented(*args, sigma)
    rs = O.raw_sums(x, y, wx, wy, ptr_x, ptr_y, sigma)
    # mixed-sign weights cancel: judge against the sums of |weight| products
    rs_abs = O.raw_sums(x, y, np.abs(wx), np.abs(wy), ptr_x, ptr_y, sigma)
    for got, k in zip((Kxx, Kyy, Kxy), range(3)):
        ref = rs.K[:, k]
        scale = rs_abs.K[:, k]
        assert np.all(np.abs(_np(got) - ref) <= K_TOL * scale + 1e-30), k
    gl = rng.uniform(0.5, 1.5, len(sizes[0]))
    gx, gy, gwx, gwy, gs = C.kde_mmd_backward_segmented(*args, _cuda(gl, dev, dtype=torch.float64),
                                                        sigma)
    rx, ry, rwx, rwy, rs_ = O.legacy_backward_segmented(x, y, wx, wy, ptr_x, ptr_y, gl, sigma)
    assert_grad(_np(gx), rx, "gx")
    assert_grad(_np(gy), ry, "gy")
    assert_grad(_np(gwx), rwx, "gwx")
    assert_grad(_np(gwy), rwy, "gwy")
    assert_grad(_np(gs), rs_, "gsigma")


def test_legacy_dense_forward_matches_oracle(cuda_device):
    from rapidalign_b200 import _cuda as C
    rng = np.random.default_rng(7)
    B, Nx, Ny, D = 5, 90, 70, 3
    x = rng.standard_normal((B, Nx, D)).astype(np.float32)
    y = rng.standard_normal((B, Ny, D)).astype(np.float32)
    wx = rng.random((B, Nx)).astype(np.float32)
    wy = rng.random((B, Ny)).astype(np.float32)
    mx = rng.random((B, Nx)) < 0.7
    my = rng.random((B, Ny)) < 0.6
    mx[3] = False  # an empty row
    dev = cuda_device
    K = C.kde_mmd_forward(*[_cuda(v, dev) for v in (x, y, wx, wy)], _cuda(mx, dev),
                          _cuda(my, dev), 0.25)
    ref = O.legacy_forward_dense(x, y, wx, wy, mx, my, 0.25)
    for got, r in zip(K, ref):
        assert np.allclose(_np(got), r, rtol=K_TOL * 5, atol=1e-12)


def test_large_pair_with_column_splits(cuda_device):
    """A pair big enough that its row tiles are split over several items."""
    import rapidalign_b200 as ra
    rng = np.random.default_rng(8)
    n, m = 9000, 8800
    x, y, ptr_x, ptr_y = _ragged(rng, [n], [m], 3)
    dev = cuda_device
    xt, yt = _cuda(x, dev, True), _cuda(y, dev, True)
    loss, Kxx, Kyy, Kxy = ra.pyg_kde_mmd_loss(xt, yt, src_ptr=_cuda(ptr_x, dev),
                                              tgt_ptr=_cuda(ptr_y, dev), sigma=0.25)
    loss.sum().backward()
    r = O.pyg_kde_mmd_loss(x, y, ptr_x, ptr_y, sigma=0.25, center=True,
                           upstream=[np.ones(1), np.zeros(1), np.zeros(1), np.zeros(1)])
    assert_k(_np(Kxx), r.Kxx)
    assert_k(_np(Kxy), r.Kxy)
    assert_loss(_np(loss), r.loss, r.Kxx, r.Kyy)
    assert_grad(_np(xt.grad), r.grad_x)
    assert_grad(_np(yt.grad), r.grad_y)


def test_deterministic_sums(cuda_device):
    import rapidalign_b200 as ra
    rng = np.random.default_rng(9)
    x, y, ptr_x, ptr_y = _ragged(rng, [500, 1200, 77], [480, 1250, 90], 3)
    dev = cuda_device
    args = dict(src_ptr=_cuda(ptr_x, dev), tgt_ptr=_cuda(ptr_y, dev), sigma=0.25)
    a = ra.pyg_kde_mmd_loss(_cuda(x, dev, True), _cuda(y, dev), **args)
    b = ra.pyg_kde_mmd_loss(_cuda(x, dev, True), _cuda(y, dev), **args)
    with torch.no_grad():
        c = ra.pyg_kde_mmd_loss(_cuda(x, dev), _cuda(y, dev), **args)
    for u, v, w in zip(a, b, c):
        assert torch.equal(u, v)  # bitwise repeatable
        assert torch.allclose(u, w, rtol=1e-6, atol=0)  # no-grad kernel agrees


def test_deterministic_mode_gradients_are_bitwise_repeatable(cuda_device):
    """torch.use_deterministic_algorithms(True) selects the deterministic mode:
    K, losses and every gradient bitwise equal across runs, and equal to the
    default mode's within the parity bars (D <= 3: both orientations, rows
    only, no atomic additions; a big pair with column tiles of many items)."""
    import rapidalign_b200 as ra
    rng = np.random.default_rng(10)
    x, y, ptr_x, ptr_y = _ragged(rng, [500, 1200, 77, 5000], [480, 1250, 90, 4800], 3)
    wx = rng.uniform(0.2, 1.0, x.shape[0]).astype(np.float32)
    dev = cuda_device
    args = dict(src_ptr=_cuda(ptr_x, dev), tgt_ptr=_cuda(ptr_y, dev), sigma=0.25)

    def run():
        xs, ys, ws = _cuda(x, dev, True), _cuda(y, dev, True), _cuda(wx, dev, True)
        outs = ra.pyg_kde_mmd_loss(xs, ys, src_w=ws, **args)
        (outs[0].sum() + 0.5 * outs[3].sum()).backward()
        return [o.detach() for o in outs] + [xs.grad, ys.grad, ws.grad]

    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(True)
    try:
        a, b = run(), run()
    finally:
        torch.use_deterministic_algorithms(prev)
    for u, v in zip(a, b):
        assert torch.equal(u, v)
    c = run()  # the default mode
    assert_loss(_np(a[0]), _np(c[0]), _np(c[1]), _np(c[2]))
    for u, v in zip(a[1:4], c[1:4]):
        assert_k(_np(u), _np(v))
    for u, v in zip(a[4:], c[4:]):
        assert_grad(_np(u), _np(v))


def test_device_detected_errors(cuda_device):
    import rapidalign_b200 as ra
    dev = cuda_device
    x = torch.randn(10, 3, device=dev)
    with pytest.raises(ValueError, match="ptr must start at 0"):
        ra.pyg_kde_mmd_loss(x, x, src_ptr=torch.tensor([1, 10], device=dev),
                            tgt_ptr=torch.tensor([0, 10], device=dev))
    with pytest.raises(ValueError, match=r"ptr\[-1\] must equal number of nodes"):
        ra.pyg_kde_mmd_loss(x, x, src_ptr=torch.tensor([0, 9], device=dev),
                            tgt_ptr=torch.tensor([0, 10], device=dev))
    with pytest.raises(ValueError, match="positive value per segment"):
        w = torch.ones(10, device=dev)
        w[:5] = -1.0
        w[5:] = 0.0
        ra.pyg_kde_mmd_loss(x, x, src_ptr=torch.tensor([0, 5, 10], device=dev),
                            tgt_ptr=torch.tensor([0, 5, 10], device=dev), src_w=w)
    with pytest.raises(ValueError, match="weights must sum to a positive value"):
        ra.kde_mmd_loss(x, x, x_w=-torch.ones(10, device=dev))
    # a decreasing ptr whose clamped ranges would overlap (and, summed, need
    # more tiles than the points allow) is reported and stays in bounds
    n = 6400
    xb = torch.randn(n, 3, device=dev)
    bad = torch.tensor([0, n, 0, n], device=dev)
    good = torch.tensor([0, 2000, 4000, n], device=dev)
    with pytest.raises(ValueError, match="ptr offsets must match node stacks"):
        ra.pyg_kde_mmd_loss(xb, xb, src_ptr=bad, tgt_ptr=good)
    with pytest.raises(ValueError, match="sorted"):
        ra.pyg_kde_mmd_loss(x, x, src_batch=torch.tensor([0, 1] * 5, device=dev),
                            tgt_batch=torch.zeros(10, dtype=torch.long, device=dev))


def test_fp64_inputs_and_dtypes(cuda_device):
    import rapidalign_b200 as ra
    dev = cuda_device
    x = torch.randn(50, 3, dtype=torch.float64, device=dev, requires_grad=True)
    y = (x.detach() + 0.05 * torch.randn_like(x)).requires_grad_(True)
    loss, Kxx, Kyy, Kxy = ra.kde_mmd_loss(x, y, sigma=0.3)
    assert loss.dtype == torch.float64 and loss.dim() == 0
    loss.backward()
    assert x.grad.dtype == torch.float64 and x.grad.shape == x.shape


def test_split_evaluation_matches_unsplit(cuda_device):
    """One pair evaluated as two shards (emulated in one process: the second
    shard's partial sums are added by hand) equals the unsplit evaluation,
    gradients included (the all-reduce path of shard.split_pair_kde_mmd_loss)."""
    from rapidalign_b200 import _lib
    from rapidalign_b200._core import Spec, backward_sums, forward_sums
    rng = np.random.default_rng(11)
    n, m = 5000, 4700
    dev = cuda_device
    x = torch.from_numpy(rng.standard_normal((n, 3)).astype(np.float32)).to(dev)
    y = torch.from_numpy(rng.standard_normal((m, 3)).astype(np.float32)).to(dev)
    # weights that require a gradient: the backward below asks for theirs
    wx = torch.from_numpy((rng.random(n) + 0.1).astype(np.float32)).to(dev).requires_grad_(True)

    def spec(idx, cnt):
        return Spec(layout=_lib.RA_LAYOUT_DENSE, num_pairs=1, dim=3, num_x=n, num_y=m, nmax_x=n,
                    nmax_y=m, weights_x=_lib.RA_WEIGHTS_SUM, weights_y=_lib.RA_WEIGHTS_UNIFORM,
                    center=True, sigma=0.2, shard_index=idx, shard_count=cnt)

    K_ref, st_ref = forward_sums(x, y, wx, None, None, spec(0, 1), True)
    stash = {}

    def grab(f64, f32):
        stash["f64"], stash["f32"] = f64.clone(), f32.clone()

    def add(f64, f32):
        f64 += stash["f64"]
        f32 += stash["f32"]

    forward_sums(x, y, wx, None, None, spec(1, 2), True, reduce=grab)
    K_sp, st_sp = forward_sums(x, y, wx, None, None, spec(0, 2), True, reduce=add)
    assert_k(_np(K_sp), _np(K_ref))
    coef = torch.tensor([1.0, 1.0, -2.0], dtype=torch.float64, device=dev)
    need = (True, True, True, False, False)
    g_ref = backward_sums(st_ref, coef, need)
    g_sp = backward_sums(st_sp, coef, need)
    for a, b in zip(g_sp[:3], g_ref[:3]):
        assert_grad(_np(a), _np(b))


def test_mid_size_single_pair_matches_oracle(cuda_device):
    """N = M = 20000: many 64-row items and column splits of one pair."""
    import rapidalign_b200 as ra
    rng = np.random.default_rng(12)
    n = 20000
    x = rng.standard_normal((n, 3)).astype(np.float32)
    y = (x + 0.05 * rng.standard_normal((n, 3))).astype(np.float32)
    dev = cuda_device
    xt, yt = _cuda(x, dev, True), _cuda(y, dev, True)
    loss, Kxx, Kyy, Kxy = ra.kde_mmd_loss(xt, yt, sigma=0.2, center=True)
    loss.backward()
    r = O.kde_mmd_loss(x, y, sigma=0.2, center=True, upstream=[1.0, 0.0, 0.0, 0.0])
    assert_k(_np(Kxx), r.Kxx)
    assert_k(_np(Kxy), r.Kxy)
    assert_loss(_np(loss), r.loss, r.Kxx, r.Kyy)
    assert_grad(_np(xt.grad), r.grad_x)
    assert_grad(_np(yt.grad), r.grad_y)


def test_multi_chunk_dense_masked_with_weights(cuda_device):
    """Rows of several 1024-point chunks: masked holes and an unmasked-free
    tail (count < Nmax), weights, centering; every gradient."""
    import rapidalign_b200 as ra
    rng = np.random.default_rng(14)
    B, Nx, Ny, D = 3, 2600, 2300, 3
    x = rng.standard_normal((B, Nx, D)).astype(np.float32)
    y = (rng.standard_normal((B, Ny, D)) * 0.8 + 0.1).astype(np.float32)
    wx = rng.uniform(0.2, 1.0, (B, Nx)).astype(np.float32)
    wy = rng.uniform(0.2, 1.0, (B, Ny)).astype(np.float32)
    mx = rng.random((B, Nx)) < 0.8
    my = rng.random((B, Ny)) < 0.9
    mx[0, 1500:] = False  # count 1500: the last chunk of the row is padding
    my[2, 1100:] = False
    dev = cuda_device
    xt, yt = _cuda(x, dev, True), _cuda(y, dev, True)
    wxt, wyt = _cuda(wx, dev, True), _cuda(wy, dev, True)
    outs = ra.kde_mmd_loss_dense(xt, yt, _cuda(mx, dev), _cuda(my, dev), x_w=wxt, y_w=wyt,
                                 sigma=0.3, center=True)
    up = [rng.uniform(0.5, 1.5, B) for _ in range(4)]
    total = sum((torch.as_tensor(u, device=dev) * o.double()).sum() for u, o in zip(up, outs))
    total.backward()
    r = O.kde_mmd_loss_dense(x, y, mx, my, wx, wy, sigma=0.3, center=True, upstream=up)
    assert_k(_np(outs[1]), r.Kxx)
    assert_k(_np(outs[2]), r.Kyy)
    assert_k(_np(outs[3]), r.Kxy)
    assert_loss(_np(outs[0]), r.loss, r.Kxx, r.Kyy)
    assert_grad(_np(xt.grad), r.grad_x, "grad_x")
    assert_grad(_np(yt.grad), r.grad_y, "grad_y")
    assert_grad(_np(wxt.grad), r.grad_wx, "grad_wx")
    assert_grad(_np(wyt.grad), r.grad_wy, "grad_wy")


@pytest.mark.parametrize("d", [5, 16])
def test_multi_chunk_generic_dims(d, cuda_device):
    """Generic-D layout with pairs of several chunks next to tiny ones."""
    import rapidalign_b200 as ra
    rng = np.random.default_rng(15 + d)
    x, y, ptr_x, ptr_y = _ragged(rng, [3100, 3, 0, 1500], [2900, 1, 4, 1700], d)
    wx = rng.uniform(0.2, 1.0, x.shape[0]).astype(np.float32)
    wy = rng.uniform(0.2, 1.0, y.shape[0]).astype(np.float32)
    dev = cuda_device
    xt, yt = _cuda(x, dev, True), _cuda(y, dev, True)
    wxt, wyt = _cuda(wx, dev, True), _cuda(wy, dev, True)
    sigma = 0.2 * np.sqrt(d)
    outs = ra.pyg_kde_mmd_loss(xt, yt, src_ptr=_cuda(ptr_x, dev), tgt_ptr=_cuda(ptr_y, dev),
                               src_w=wxt, tgt_w=wyt, sigma=sigma, center=True)
    up = [rng.uniform(0.5, 1.5, 4) for _ in range(4)]
    total = sum((torch.as_tensor(u, device=dev) * o.double()).sum() for u, o in zip(up, outs))
    total.backward()
    r = O.pyg_kde_mmd_loss(x, y, ptr_x, ptr_y, wx, wy, sigma=sigma, center=True, upstream=up)
    assert_k(_np(outs[1]), r.Kxx)
    assert_k(_np(outs[2]), r.Kyy)
    assert_k(_np(outs[3]), r.Kxy)
    assert_loss(_np(outs[0]), r.loss, r.Kxx, r.Kyy)
    assert_grad(_np(xt.grad), r.grad_x, "grad_x")
    assert_grad(_np(yt.grad), r.grad_y, "grad_y")
    assert_grad(_np(wxt.grad), r.grad_wx, "grad_wx")
    assert_grad(_np(wyt.grad), r.grad_wy, "grad_wy")
