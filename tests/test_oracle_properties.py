"""Properties of the oracle itself, ported from the reference's CPU tests
(tests/test_kde_similarity.py:13-41, tests/test_kde_gradients.py:105-216)."""
import numpy as np

from oracle import oracle as O


def test_identical_zero_loss():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((32, 3))
    r = O.kde_mmd_loss(x, x, sigma=0.3, center=True)
    assert abs(r.loss) < 1e-12
    assert abs(r.Kxx - r.Kxy) < 1e-12


def test_translation_invariance():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((40, 3))
    y = x + np.array([0.5, -0.2, 0.1])
    c = O.kde_mmd_loss(x, y, sigma=0.2, center=True)
    u = O.kde_mmd_loss(x, y, sigma=0.2, center=False)
    assert abs(c.loss) < 1e-12
    assert u.loss > c.loss


def test_cosine_identical_zero():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((16, 3))
    assert abs(O.kde_mmd_loss(x, x, sigma=0.3, cosine=True).loss) < 1e-12


def _fd(f, v, eps=1e-6):
    g = np.zeros_like(v)
    it = np.nditer(v, flags=["multi_index"])
    for _ in it:
        i = it.multi_index
        vp, vm = v.copy(), v.copy()
        vp[i] += eps
        vm[i] -= eps
        g[i] = (f(vp) - f(vm)) / (2 * eps)
    return g


def test_pyg_gradients_match_finite_differences():
    """Full public-API chain rule (normalised weights, centering, cosine)."""
    rng = np.random.default_rng(3)
    ptr_x = np.array([0, 4, 9])
    ptr_y = np.array([0, 5, 8])
    x = rng.standard_normal((9, 3))
    y = rng.standard_normal((8, 3))
    wx = rng.random(9) + 0.2
    wy = rng.random(8) + 0.2
    up = [np.array([1.0, 0.5]), np.array([0.2, -0.1]), np.array([0.0, 0.3]), np.array([-0.4, 0.1])]

    for cosine in (False, True):
        def total(xx=x, yy=y, wxx=wx, wyy=wy, sg=0.4):
            r = O.pyg_kde_mmd_loss(xx, yy, ptr_x, ptr_y, wxx, wyy, sigma=sg, center=True,
                                   cosine=cosine)
            return sum(float(np.dot(u, v)) for u, v in zip(up, (r.loss, r.Kxx, r.Kyy, r.Kxy)))

        r = O.pyg_kde_mmd_loss(x, y, ptr_x, ptr_y, wx, wy, sigma=0.4, center=True,
                               cosine=cosine, upstream=up)
        np.testing.assert_allclose(r.grad_x, _fd(lambda v: total(xx=v), x), atol=1e-7)
        np.testing.assert_allclose(r.grad_y, _fd(lambda v: total(yy=v), y), atol=1e-7)
        np.testing.assert_allclose(r.grad_wx, _fd(lambda v: total(wxx=v), wx), atol=1e-7)
        np.testing.assert_allclose(r.grad_wy, _fd(lambda v: total(wyy=v), wy), atol=1e-7)
        fd_s = (total(sg=0.4 + 1e-6) - total(sg=0.4 - 1e-6)) / 2e-6
        assert abs(r.grad_sigma - fd_s) < 1e-6


def test_ragged_equals_per_pair():
    rng = np.random.default_rng(4)
    ptr_x = np.array([0, 3, 7, 7, 12])
    ptr_y = np.array([0, 4, 6, 9, 9])
    x = rng.standard_normal((12, 2))
    y = rng.standard_normal((9, 2))
    a = rng.random(12)
    b = rng.random(9)
    rs = O.raw_sums(x, y, a, b, ptr_x, ptr_y, 0.35)
    for p in range(4):
        xs, ys = slice(ptr_x[p], ptr_x[p + 1]), slice(ptr_y[p], ptr_y[p + 1])
        one = O.raw_sums(x[xs], y[ys], a[xs], b[ys], [0, ptr_x[p + 1] - ptr_x[p]],
                         [0, ptr_y[p + 1] - ptr_y[p]], 0.35)
        np.testing.assert_allclose(rs.K[p], one.K[0], rtol=1e-14, atol=1e-300)
        np.testing.assert_allclose(rs.G_xy[xs], one.G_xy, rtol=1e-13, atol=1e-300)


def test_thread_count_does_not_change_results():
    rng = np.random.default_rng(5)
    ptr = np.array([0, 50, 130])
    x = rng.standard_normal((130, 3))
    y = rng.standard_normal((130, 3))
    a = rng.random(130)
    r1 = O.raw_sums(x, y, a, a, ptr, ptr, 0.25, nthreads=1)
    r4 = O.raw_sums(x, y, a, a, ptr, ptr, 0.25, nthreads=4)
    assert np.array_equal(r1.K, r4.K) and np.array_equal(r1.G_xx, r4.G_xx)


def test_rows_match_full():
    rng = np.random.default_rng(6)
    x = rng.standard_normal((60, 3))
    y = rng.standard_normal((50, 3))
    a = rng.random(60)
    b = rng.random(50)
    full = O.raw_sums(x, y, a, b, [0, 60], [0, 50], 0.3)
    rows = np.array([0, 7, 59])
    ss, sG, cs, cG = O.rows_sums(0, x, y, a, b, 0.3, rows)
    np.testing.assert_allclose(ss, full.s_xx[rows], rtol=1e-14)
    np.testing.assert_allclose(cG, full.G_xy[rows], rtol=1e-13)
