"""CPU fp64 oracle for the KDE/MMD hot path.

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, by the smoke check in
``__graft_entry__.py`` and by the CPU-baseline leg of ``bench.py``, always as
the reference the CUDA path is compared with.  The product package (``rapidalign_b200``) never imports it.

The heavy O(N*M) part is ``kde_oracle.c`` (a plain-C, double-precision
restatement of ``rapidalign/kde_gradients.py:32-193``) loaded through ctypes.
This module adds, in numpy fp64, the parts of the public API that the
reference gets from PyTorch autograd on its CPU path:

* weight normalisation, ``rapidalign/kde.py:20-27`` (single pair),
  ``kde.py:169-199`` (ragged) and ``kde.py:115-121`` (dense, clamped);
* weighted-centroid centering, ``kde.py:77-81``, ``kde.py:202-208``,
  ``kde.py:246-253``;
* the MMD and cosine losses, ``kde.py:103-107`` / ``kde.py:368-371``;
* the backward of all of the above for arbitrary upstream gradients on the
  four outputs ``(loss, Kxx, Kyy, Kxy)``.

It also restates the three legacy extension ops of ``csrc/bindings.cpp:34-71``
(raw weights, no centering): ``kde_similarity.cu:84-192`` (dense masked
forward), ``:283-381`` (segmented forward) and ``:607-712`` (segmented
backward), and the CPU branch of ``rapidalign/autograd_kde.py:16-117``.

The oracle is pinned against golden vectors produced by running the reference
itself in float64 (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(_HERE, "kde_oracle.c")
_LIB_DIR = os.path.join(_HERE, "_build")
_LIB_PATH = os.path.join(_LIB_DIR, "libkde_oracle.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile ``kde_oracle.c`` into ``oracle/_build/libkde_oracle.so``."""
    if (not force and os.path.exists(_LIB_PATH)
            and os.path.getmtime(_LIB_PATH) >= os.path.getmtime(_SRC)):
        return _LIB_PATH
    os.makedirs(_LIB_DIR, exist_ok=True)
    tmp = _LIB_PATH + f".tmp{os.getpid()}"
    cmd = ["gcc", "-O3", "-fopenmp", "-fPIC", "-shared", "-o", tmp, _SRC, "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, _LIB_PATH)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        path = build()
        lib = ctypes.CDLL(path)
        dp = ctypes.POINTER(ctypes.c_double)
        lp = ctypes.POINTER(ctypes.c_int64)
        lib.ra_oracle_segmented.restype = ctypes.c_int
        lib.ra_oracle_segmented.argtypes = [
            ctypes.c_int64, ctypes.c_int, dp, dp, dp, dp, lp, lp, ctypes.c_double, ctypes.c_int,
            dp, dp, dp, dp, dp, dp, dp, dp, dp, dp]
        lib.ra_oracle_rows.restype = ctypes.c_int
        lib.ra_oracle_rows.argtypes = [
            ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, dp, dp, dp, dp,
            ctypes.c_double, ctypes.c_int64, lp, ctypes.c_int, dp, dp, dp, dp]
        _lib = lib
    return _lib


def _dp(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def _lp(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))


def _f64(a, shape_dims=None) -> np.ndarray:
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float64))
    return a


@dataclass
class RawSums:
    """Per-pair K/S sums and per-point row sums of one ragged batch (fp64)."""
    K: np.ndarray      # (P, 3): Kxx, Kyy, Kxy
    S: np.ndarray      # (P, 3): sum of w w' k r^2 over ordered pairs
    s_xx: np.ndarray   # (NX,)
    s_xy: np.ndarray   # (NX,)
    G_xx: np.ndarray   # (NX, D)
    G_xy: np.ndarray   # (NX, D)
    s_yy: np.ndarray   # (NY,)
    s_yx: np.ndarray   # (NY,)
    G_yy: np.ndarray   # (NY, D)
    G_yx: np.ndarray   # (NY, D)


def raw_sums(x, y, a, b, ptr_x, ptr_y, sigma: float, nthreads: int = 0) -> RawSums:
    """Restates kde_gradients.py:39-132 for every pair of a ptr-segmented batch."""
    x = _f64(x)
    y = _f64(y)
    a = _f64(a).reshape(-1)
    b = _f64(b).reshape(-1)
    ptr_x = np.ascontiguousarray(np.asarray(ptr_x, dtype=np.int64))
    ptr_y = np.ascontiguousarray(np.asarray(ptr_y, dtype=np.int64))
    P = ptr_x.size - 1
    D = x.shape[1] if x.ndim == 2 else y.shape[1]
    NX, NY = x.shape[0], y.shape[0]
    x = x.reshape(NX, D)
    y = y.reshape(NY, D)
    out = RawSums(
        K=np.zeros((max(P, 0), 3)), S=np.zeros((max(P, 0), 3)),
        s_xx=np.zeros(NX), s_xy=np.zeros(NX), G_xx=np.zeros((NX, D)), G_xy=np.zeros((NX, D)),
        s_yy=np.zeros(NY), s_yx=np.zeros(NY), G_yy=np.zeros((NY, D)), G_yx=np.zeros((NY, D)))
    if P <= 0:
        return out
    # ctypes cannot take a pointer to a zero-length array's data safely: pad.
    def nz(arr, shape):
        return arr if arr.size else np.zeros(shape)
    xs, ys = nz(x, (1, D)), nz(y, (1, D))
    as_, bs = nz(a, (1,)), nz(b, (1,))
    bufs = [nz(out.s_xx, (1,)), nz(out.s_xy, (1,)), nz(out.G_xx, (1, D)), nz(out.G_xy, (1, D)),
            nz(out.s_yy, (1,)), nz(out.s_yx, (1,)), nz(out.G_yy, (1, D)), nz(out.G_yx, (1, D))]
    rc = _load().ra_oracle_segmented(
        P, D, _dp(xs), _dp(ys), _dp(as_), _dp(bs), _lp(ptr_x), _lp(ptr_y), float(sigma),
        int(nthreads), _dp(out.K), _dp(out.S), *[_dp(t) for t in bufs])
    if rc != 0:
        raise ValueError("oracle: invalid arguments")
    return out


def rows_sums(side: int, x, y, a, b, sigma: float, rows, nthreads: int = 0):
    """Row sums of selected rows of ONE pair: (self_s, self_G, cross_s, cross_G)."""
    x, y = _f64(x), _f64(y)
    a, b = _f64(a).reshape(-1), _f64(b).reshape(-1)
    rows = np.ascontiguousarray(np.asarray(rows, dtype=np.int64))
    D = x.shape[1]
    R = rows.size
    ss, cs = np.zeros(R), np.zeros(R)
    sG, cG = np.zeros((R, D)), np.zeros((R, D))
    rc = _load().ra_oracle_rows(side, D, x.shape[0], y.shape[0], _dp(x), _dp(y), _dp(a), _dp(b),
                                float(sigma), R, _lp(rows), int(nthreads), _dp(ss), _dp(sG),
                                _dp(cs), _dp(cG))
    if rc != 0:
        raise ValueError("oracle: invalid arguments")
    return ss, sG, cs, cG


# --------------------------------------------------------------------------
# segment helpers (numpy restatements of kde.py:124-208)
# --------------------------------------------------------------------------

def _seg_ids(ptr: np.ndarray) -> np.ndarray:
    counts = np.diff(ptr)
    return np.repeat(np.arange(ptr.size - 1), counts)


def _seg_sum(values: np.ndarray, ptr: np.ndarray) -> np.ndarray:
    P = ptr.size - 1
    out = np.zeros((P,) + values.shape[1:])
    if values.shape[0]:
        np.add.at(out, _seg_ids(ptr), values)
    return out


def ptr_from_batch(batch) -> np.ndarray:
    """kde.py:142-156: ptr from a sorted batch vector."""
    batch = np.asarray(batch, dtype=np.int64)
    if batch.size == 0:
        return np.zeros(1, dtype=np.int64)
    if np.any(batch[:-1] > batch[1:]):
        raise ValueError("batch indices must be sorted for contiguous blocks")
    P = int(batch[-1]) + 1
    counts = np.bincount(batch, minlength=P)
    ptr = np.zeros(P + 1, dtype=np.int64)
    ptr[1:] = np.cumsum(counts)
    return ptr


@dataclass
class LossResult:
    loss: np.ndarray
    Kxx: np.ndarray
    Kyy: np.ndarray
    Kxy: np.ndarray
    grad_x: Optional[np.ndarray] = None
    grad_y: Optional[np.ndarray] = None
    grad_wx: Optional[np.ndarray] = None
    grad_wy: Optional[np.ndarray] = None
    grad_sigma: Optional[float] = None


def _loss_and_coeffs(K: np.ndarray, cosine: bool, eps: float, upstream):
    """Loss from K (kde.py:103-107) and the coefficients dL_total/dK per pair."""
    Kxx, Kyy, Kxy = K[:, 0], K[:, 1], K[:, 2]
    if cosine:
        prod = Kxx * Kyy
        c = np.maximum(prod, eps)
        den = np.sqrt(c)
        loss = 1.0 - Kxy / den
    else:
        loss = Kxx + Kyy - 2.0 * Kxy
    if upstream is None:
        return loss, None
    g_loss, g_kxx, g_kyy, g_kxy = [np.broadcast_to(np.asarray(u, dtype=np.float64), loss.shape)
                                   for u in upstream]
    if cosine:
        # d/dK of 1 - Kxy / sqrt(clamp_min(Kxx*Kyy, eps)); clamp passes grad where prod >= eps
        pass_through = (prod >= eps).astype(np.float64)
        dden = Kxy / (den * den)  # dL/dden
        dprod = dden * 0.5 / den * pass_through
        cxx = g_kxx + g_loss * dprod * Kyy
        cyy = g_kyy + g_loss * dprod * Kxx
        cxy = g_kxy + g_loss * (-1.0 / den)
    else:
        cxx = g_kxx + g_loss
        cyy = g_kyy + g_loss
        cxy = g_kxy - 2.0 * g_loss
    return loss, np.stack([cxx, cyy, cxy], axis=1)


def _ragged_core(x, y, ptr_x, ptr_y, a, b, w_x, w_y, sigma, center, cosine, eps, upstream,
                 nthreads, weight_mode):
    """Shared forward/backward for the ragged and single-pair public APIs.

    weight_mode: 'sum' (a = w / sum w), 'uniform' (w is None), 'raw' (a = w)."""
    x, y = _f64(x), _f64(y)
    D = x.shape[1]
    if center:
        mu_x = _seg_sum(a[:, None] * x, ptr_x)
        mu_y = _seg_sum(b[:, None] * y, ptr_y)
        xt = x - mu_x[_seg_ids(ptr_x)]
        yt = y - mu_y[_seg_ids(ptr_y)]
    else:
        xt, yt = x, y
    rs = raw_sums(xt, yt, a, b, ptr_x, ptr_y, sigma, nthreads)
    loss, coef = _loss_and_coeffs(rs.K, cosine, eps, upstream)
    res = LossResult(loss=loss, Kxx=rs.K[:, 0].copy(), Kyy=rs.K[:, 1].copy(),
                     Kxy=rs.K[:, 2].copy())
    if coef is None:
        return res
    inv_s2 = 1.0 / (sigma * sigma)
    sx, sy = _seg_ids(ptr_x), _seg_ids(ptr_y)
    cxx, cyy, cxy = coef[:, 0], coef[:, 1], coef[:, 2]
    # dL/dx~ and dL/da (direct), kde_gradients.py:98-113 generalised to any coefficients
    gxt = -inv_s2 * a[:, None] * (2.0 * cxx[sx][:, None] * rs.G_xx + cxy[sx][:, None] * rs.G_xy)
    gyt = -inv_s2 * b[:, None] * (2.0 * cyy[sy][:, None] * rs.G_yy + cxy[sy][:, None] * rs.G_yx)
    ga = 2.0 * cxx[sx] * rs.s_xx + cxy[sx] * rs.s_xy
    gb = 2.0 * cyy[sy] * rs.s_yy + cxy[sy] * rs.s_yx
    if center:
        Rx = _seg_sum(gxt, ptr_x)
        Ry = _seg_sum(gyt, ptr_y)
        gx = gxt - a[:, None] * Rx[sx]
        gy = gyt - b[:, None] * Ry[sy]
        ga = ga - np.einsum("nd,nd->n", x, Rx[sx])
        gb = gb - np.einsum("nd,nd->n", y, Ry[sy])
    else:
        gx, gy = gxt, gyt
    res.grad_x, res.grad_y = gx, gy
    if weight_mode == "sum":
        Wx = _seg_sum(w_x, ptr_x)
        Wy = _seg_sum(w_y, ptr_y)
        res.grad_wx = (ga - _seg_sum(a * ga, ptr_x)[sx]) / Wx[sx]
        res.grad_wy = (gb - _seg_sum(b * gb, ptr_y)[sy]) / Wy[sy]
    elif weight_mode == "raw":
        res.grad_wx, res.grad_wy = ga, gb
    # sigma: dK/dsigma = S / sigma^3 (kde_gradients.py:115-123)
    res.grad_sigma = float(np.sum(cxx * rs.S[:, 0] + cyy * rs.S[:, 1] + cxy * rs.S[:, 2])
                           / sigma ** 3)
    return res


def _normalise_ragged(w, ptr, n):
    """kde.py:169-199."""
    if w is None:
        counts = np.diff(ptr).astype(np.float64)
        per = np.zeros(counts.size)
        per[counts > 0] = 1.0 / counts[counts > 0]
        return per[_seg_ids(ptr)], None, "uniform"
    w = _f64(w).reshape(-1)
    if w.size != n:
        raise ValueError("weights length must equal number of nodes")
    sums = _seg_sum(w, ptr)[_seg_ids(ptr)]
    if np.any(sums <= 0):
        raise ValueError("weights must sum to a positive value per segment")
    return w / sums, w, "sum"


def pyg_kde_mmd_loss(src_pos, tgt_pos, src_ptr, tgt_ptr, src_w=None, tgt_w=None, sigma=0.2,
                     center=True, cosine=False, eps=1e-8, upstream=None,
                     nthreads: int = 0) -> LossResult:
    """Oracle for kde.py:302-428 (values and, given upstream grads, all grads)."""
    src_ptr = np.asarray(src_ptr, dtype=np.int64)
    tgt_ptr = np.asarray(tgt_ptr, dtype=np.int64)
    a, w_x, mode_x = _normalise_ragged(src_w, src_ptr, np.asarray(src_pos).shape[0])
    b, w_y, mode_y = _normalise_ragged(tgt_w, tgt_ptr, np.asarray(tgt_pos).shape[0])
    mode = "sum" if (mode_x == "sum" or mode_y == "sum") else "uniform"
    if mode == "sum":
        w_x = w_x if w_x is not None else np.ones(np.asarray(src_pos).shape[0])
        w_y = w_y if w_y is not None else np.ones(np.asarray(tgt_pos).shape[0])
    res = _ragged_core(src_pos, tgt_pos, src_ptr, tgt_ptr, a, b, w_x, w_y, float(sigma), center,
                       cosine, eps, upstream, nthreads, mode)
    if mode_x == "uniform":
        res.grad_wx = None
    if mode_y == "uniform":
        res.grad_wy = None
    return res


def kde_mmd_loss(x, y, x_w=None, y_w=None, sigma=0.2, center=True, cosine=False, eps=1e-8,
                 upstream=None, nthreads: int = 0) -> LossResult:
    """Oracle for kde.py:39-109 (one pair; results are 0-d)."""
    x = _f64(x)
    y = _f64(y)
    ptr_x = np.array([0, x.shape[0]], dtype=np.int64)
    ptr_y = np.array([0, y.shape[0]], dtype=np.int64)
    if x_w is not None and np.sum(np.asarray(x_w, dtype=np.float64)) <= 0:
        raise ValueError("weights must sum to a positive value")
    if y_w is not None and np.sum(np.asarray(y_w, dtype=np.float64)) <= 0:
        raise ValueError("weights must sum to a positive value")
    a = (np.full(x.shape[0], 1.0 / max(x.shape[0], 1)) if x_w is None
         else _f64(x_w) / np.sum(_f64(x_w)))
    b = (np.full(y.shape[0], 1.0 / max(y.shape[0], 1)) if y_w is None
         else _f64(y_w) / np.sum(_f64(y_w)))
    wx = _f64(x_w) if x_w is not None else np.ones(x.shape[0])
    wy = _f64(y_w) if y_w is not None else np.ones(y.shape[0])
    res = _ragged_core(x, y, ptr_x, ptr_y, a, b, wx, wy, float(sigma), center, cosine, eps,
                       upstream, nthreads, "sum")
    if x_w is None:
        res.grad_wx = None
    if y_w is None:
        res.grad_wy = None
    for f in ("loss", "Kxx", "Kyy", "Kxy"):
        setattr(res, f, getattr(res, f)[0])
    return res


def kde_mmd_loss_dense(x, y, mask_x, mask_y, x_w=None, y_w=None, sigma=0.2, center=True,
                       cosine=False, eps=1e-8, upstream=None, nthreads: int = 0) -> LossResult:
    """Oracle for kde.py:211-299 as computed by its CUDA branch (masked sums)."""
    x, y = _f64(x), _f64(y)
    B, NXm, D = x.shape
    NYm = y.shape[1]
    mx = np.asarray(mask_x, dtype=bool)
    my = np.asarray(mask_y, dtype=bool)
    wx_in = mx.astype(np.float64) if x_w is None else _f64(x_w) * mx
    wy_in = my.astype(np.float64) if y_w is None else _f64(y_w) * my
    Sx = np.maximum(wx_in.sum(1), 1e-8)
    Sy = np.maximum(wy_in.sum(1), 1e-8)
    a = (wx_in / Sx[:, None]).reshape(-1)
    b = (wy_in / Sy[:, None]).reshape(-1)
    ptr_x = np.arange(B + 1, dtype=np.int64) * NXm
    ptr_y = np.arange(B + 1, dtype=np.int64) * NYm
    xf = x.reshape(-1, D)
    yf = y.reshape(-1, D)
    res = _ragged_core(xf, yf, ptr_x, ptr_y, a, b, None, None, float(sigma), center, cosine, eps,
                       upstream, nthreads, "raw")
    if upstream is not None:
        # x_proc = (x - mu) * mask: masked rows get no gradient (a=0 there already,
        # and the centering term is multiplied by the mask)
        res.grad_x = (res.grad_x * mx.reshape(-1)[:, None]).reshape(B, NXm, D)
        res.grad_y = (res.grad_y * my.reshape(-1)[:, None]).reshape(B, NYm, D)
        ga = res.grad_wx.reshape(B, NXm)
        gb = res.grad_wy.reshape(B, NYm)
        a2, b2 = a.reshape(B, NXm), b.reshape(B, NYm)

        def wgrad(g, aa, m, S, raw_sum):
            unclamped = (raw_sum > 1e-8)[:, None]
            proj = (g - (aa * g).sum(1, keepdims=True)) / S[:, None]
            return np.where(unclamped, proj, g / S[:, None]) * m

        res.grad_wx = wgrad(ga, a2, mx, Sx, wx_in.sum(1)) if x_w is not None else None
        res.grad_wy = wgrad(gb, b2, my, Sy, wy_in.sum(1)) if y_w is not None else None
    return res


# --------------------------------------------------------------------------
# legacy extension ops (csrc/bindings.cpp:34-71) and the autograd op
# --------------------------------------------------------------------------

def legacy_forward_segmented(x, y, w_x, w_y, ptr_x, ptr_y, sigma):
    """kde_similarity.cu:283-381: raw-weight K sums per pair."""
    rs = raw_sums(x, y, w_x, w_y, ptr_x, ptr_y, sigma)
    return rs.K[:, 0].copy(), rs.K[:, 1].copy(), rs.K[:, 2].copy()


def legacy_forward_dense(x, y, w_x, w_y, mask_x, mask_y, sigma):
    """kde_similarity.cu:84-192: masked raw-weight K sums per batch row."""
    x, y = _f64(x), _f64(y)
    B, NXm, D = x.shape
    NYm = y.shape[1]
    a = (_f64(w_x) * np.asarray(mask_x, dtype=bool)).reshape(-1)
    b = (_f64(w_y) * np.asarray(mask_y, dtype=bool)).reshape(-1)
    ptr_x = np.arange(B + 1, dtype=np.int64) * NXm
    ptr_y = np.arange(B + 1, dtype=np.int64) * NYm
    rs = raw_sums(x.reshape(-1, D), y.reshape(-1, D), a, b, ptr_x, ptr_y, sigma)
    return rs.K[:, 0].copy(), rs.K[:, 1].copy(), rs.K[:, 2].copy()


def legacy_backward_segmented(x, y, w_x, w_y, ptr_x, ptr_y, grad_loss, sigma):
    """kde_similarity.cu:607-712: grads of sum_p grad_loss[p] * (Kxx+Kyy-2Kxy)[p]."""
    a = _f64(w_x).reshape(-1)
    b = _f64(w_y).reshape(-1)
    ptr_x = np.asarray(ptr_x, dtype=np.int64)
    ptr_y = np.asarray(ptr_y, dtype=np.int64)
    rs = raw_sums(x, y, a, b, ptr_x, ptr_y, sigma)
    gl = _f64(grad_loss).reshape(-1)
    sx, sy = _seg_ids(ptr_x), _seg_ids(ptr_y)
    scale = 2.0 / (sigma * sigma)
    gx = gl[sx][:, None] * (-scale * a[:, None] * rs.G_xx + scale * a[:, None] * rs.G_xy)
    gy = gl[sy][:, None] * (-scale * b[:, None] * rs.G_yy + scale * b[:, None] * rs.G_yx)
    gwx = gl[sx] * (2.0 * rs.s_xx - 2.0 * rs.s_xy)
    gwy = gl[sy] * (2.0 * rs.s_yy - 2.0 * rs.s_yx)
    gsig = gl * (rs.S[:, 0] + rs.S[:, 1] - 2.0 * rs.S[:, 2]) / sigma ** 3
    return gx, gy, gwx, gwy, gsig


def segmented_kde_loss(x, y, w_x, w_y, ptr_x, ptr_y, sigma, grad_loss=None):
    """autograd_kde.py:16-129 (raw weights, no centering): per-pair losses and,
    given grad_loss, grads (x, y, w_x, w_y, sigma-total)."""
    Kxx, Kyy, Kxy = legacy_forward_segmented(x, y, w_x, w_y, ptr_x, ptr_y, sigma)
    loss = Kxx + Kyy - 2.0 * Kxy
    if grad_loss is None:
        return loss, None
    gx, gy, gwx, gwy, gsig = legacy_backward_segmented(x, y, w_x, w_y, ptr_x, ptr_y,
                                                       grad_loss, sigma)
    return loss, (gx, gy, gwx, gwy, float(np.sum(gsig)))


# ---------------------------------------------------------------------------
# pairwise-distance spectrum loss (rapidalign/algorithms.py:19-90)
# ---------------------------------------------------------------------------

def _groups(points: np.ndarray, batch) -> list:
    """algorithms.py:19-34: the point sets of the sorted unique batch ids (the
    points of one id keep their order)."""
    if batch is None:
        return [np.arange(points.shape[0])]
    batch = np.asarray(batch).reshape(-1)
    return [np.nonzero(batch == g)[0] for g in np.unique(batch)]


def _triu_dists(p: np.ndarray):
    """algorithms.py:37-44: distances of all pairs i < j (row-major upper
    triangle), with the pair indices, before sorting."""
    n = p.shape[0]
    if n < 2:
        return np.zeros(0), np.zeros(0, dtype=np.int64), np.zeros(0, dtype=np.int64)
    i, j = np.triu_indices(n, k=1)
    d = np.sqrt(((p[i] - p[j]) ** 2).sum(axis=1))
    return d, i, j


def pairwise_distance_loss(src, tgt, src_batch=None, tgt_batch=None, reduction="mean",
                           upstream=None):
    """algorithms.py:54-90 in float64: per group, the sorted pair distances of
    src and tgt, the shorter padded with zeros at the end, their mean squared
    difference; then the reduction.  With ``upstream`` (dL/d of the returned
    value, shape of the result) also returns (grad_src, grad_tgt): the sort
    passes each position's gradient to its pair, the norm's gradient at a
    zero distance is 0 (as torch.linalg.norm's)."""
    src = _f64(src)
    tgt = _f64(tgt)
    gs, gt = _groups(src, src_batch), _groups(tgt, tgt_batch)
    if len(gs) != len(gt):
        raise ValueError("src and tgt batch counts must match")
    losses = []
    parts = []
    for a, b in zip(gs, gt):
        ds, si, sj = _triu_dists(src[a])
        dt, ti, tj = _triu_dists(tgt[b])
        os_, ot = np.argsort(ds, kind="stable"), np.argsort(dt, kind="stable")
        L = max(ds.size, dt.size)
        sv = np.zeros(L)
        tv = np.zeros(L)
        sv[:ds.size] = ds[os_]
        tv[:dt.size] = dt[ot]
        losses.append(np.mean((sv - tv) ** 2) if L else np.nan)
        parts.append((a, b, ds, si, sj, os_, dt, ti, tj, ot, sv, tv, L))
    losses = np.array(losses)
    if reduction == "mean":
        out = losses.mean()
    elif reduction == "sum":
        out = losses.sum()
    elif reduction == "none":
        out = losses
    else:
        raise ValueError(f"Unsupported reduction: {reduction}")
    if upstream is None:
        return out
    up = np.broadcast_to(np.asarray(upstream, dtype=np.float64), losses.shape) \
        if reduction == "none" else np.full(losses.shape, float(upstream))
    if reduction == "mean":
        up = up / len(losses)
    grad_src = np.zeros_like(src)
    grad_tgt = np.zeros_like(tgt)
    for g, (a, b, ds, si, sj, os_, dt, ti, tj, ot, sv, tv, L) in enumerate(parts):
        if L == 0:
            continue
        gpos = 2.0 * (sv - tv) / L * up[g]  # d loss / d sv (and minus for tv)
        for pts, grad, d, pi, pj, order, sign, cnt in (
                (src[a], grad_src, ds, si, sj, os_, 1.0, ds.size),
                (tgt[b], grad_tgt, dt, ti, tj, ot, -1.0, dt.size)):
            if cnt == 0:
                continue
            gd = np.zeros(cnt)
            gd[order] = sign * gpos[:cnt]
            with np.errstate(invalid="ignore", divide="ignore"):
                coef = np.where(d > 0, gd / d, 0.0)
            vec = coef[:, None] * (pts[pi] - pts[pj])
            idx = a if sign > 0 else b
            np.add.at(grad, idx[pi], vec)
            np.add.at(grad, idx[pj], -vec)
    return out, grad_src, grad_tgt
