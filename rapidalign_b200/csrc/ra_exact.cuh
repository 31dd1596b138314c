// ra_exact.cuh -- float64 verification path: the closed-form sums and
// gradients of the raw-weight MMD (rapidalign/kde_gradients.py:39-193) and
// the dense kernel / difference matrices of one pair (kde_gradients.py:32-36).
//
// These mirror the reference's float64 verification helpers, so every term
// is evaluated in double precision with exp(), in a plain direct loop: one
// thread per point of x or y walks its own cloud and the other cloud of its
// pair.  The work is O(N^2 D) per pair and meant for the small problems such
// helpers are used on; the fast fused path lives in the tile kernels.
//
// Per point i (cloud A, partner cloud B, weights w, s2 = 2 / sigma^2):
//   ss = sum_{j in A} w_j k_ij,  gs = sum_{j in A} w_j k_ij (p_i - p_j),
//   sc = sum_{j in B} w_j k_ij,  gc = sum_{j in B} w_j k_ij (p_i - q_j),
//   rs, rc = the same sums with k r^2 (for d/dsigma);
//   dL/dp_i = -s2 w_i gs + s2 w_i gc,   dL/dw_i = 2 ss - 2 sc
// (kde_gradients.py:98-118; the y side is the same formula with the roles
// swapped, kde_gradients.py:104-111).  A second kernel, one CTA per pair,
// sums w_i ss, w_i sc, w_i rs, w_i rc over the pair's points in a fixed
// order: Kxx, Kyy, Kxy and dL/dsigma (kde_gradients.py:120-127).
#pragma once

#include "ra_common.cuh"

namespace ra {

constexpr int kExactMaxD = 256;
constexpr int kExactChunk = 32;

struct ExactArgs {
  int64_t P, NX, NY;
  int D;
  double sigma;
  const double *x, *y, *w_x, *w_y;
  const int64_t *ptr_x, *ptr_y;
  double *grad_x, *grad_y, *grad_wx, *grad_wy;  // nullable
  double *work;  // [NX + NY][4]: w ss, w sc, w rs, w rc
  int *err;
};

// Pair of element `i` of a ptr array (the p with ptr[p] <= i < ptr[p + 1]).
__device__ __forceinline__ int64_t pair_of(const int64_t *ptr, int64_t P, int64_t i) {
  int64_t lo = 0, hi = P;  // ptr[lo] <= i < ptr[hi]
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (ptr[mid] <= i) lo = mid;
    else hi = mid;
  }
  return lo;
}

// ptr checks of both sides (kde.py:133-149 semantics): first 0, last N,
// non-decreasing.  One thread per entry.
__global__ void exact_check_kernel(ExactArgs A) {
  const int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (k > A.P) return;
  for (int side = 0; side < 2; ++side) {
    const int64_t *ptr = side == 0 ? A.ptr_x : A.ptr_y;
    const int64_t N = side == 0 ? A.NX : A.NY;
    if (k == 0 && ptr[0] != 0) atomicOr(A.err, (int)kErrPtrStart);
    if (k == A.P && ptr[A.P] != N) atomicOr(A.err, (int)kErrPtrEnd);
    if (k < A.P && ptr[k] > ptr[k + 1]) atomicOr(A.err, (int)kErrPtrOrder);
  }
}

__global__ void __launch_bounds__(128) exact_points_kernel(ExactArgs A) {
  const int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (g >= A.NX + A.NY) return;
  const int side = g < A.NX ? 0 : 1;
  const int64_t i = side == 0 ? g : g - A.NX;
  const int64_t *ptr_a = side == 0 ? A.ptr_x : A.ptr_y;
  const int64_t *ptr_b = side == 0 ? A.ptr_y : A.ptr_x;
  const double *pa = side == 0 ? A.x : A.y;
  const double *pb = side == 0 ? A.y : A.x;
  const double *wa = side == 0 ? A.w_x : A.w_y;
  const double *wb = side == 0 ? A.w_y : A.w_x;
  const int64_t p = pair_of(ptr_a, A.P, i);
  const int D = A.D;
  const double inv2s2 = 1.0 / (2.0 * A.sigma * A.sigma);
  const double w = wa[i], s2 = 2.0 / (A.sigma * A.sigma);
  double *gout = side == 0 ? A.grad_x : A.grad_y;
  double *wout = side == 0 ? A.grad_wx : A.grad_wy;
  const double *pi = pa + i * D;
  double ss = 0.0, sc = 0.0, rs = 0.0, rc = 0.0;
  // coordinates in chunks of 32 (the kernel values are recomputed per
  // chunk, which keeps the per-thread sums small)
  for (int dc = 0; dc < D; dc += kExactChunk) {
    const int nd = D - dc < kExactChunk ? D - dc : kExactChunk;
    double gs[kExactChunk], gc[kExactChunk];
    for (int d = 0; d < kExactChunk; ++d) gs[d] = gc[d] = 0.0;
    for (int other = 0; other < 2; ++other) {
      const double *pc = other == 0 ? pa : pb;
      const double *wc = other == 0 ? wa : wb;
      const int64_t *ptr_c = other == 0 ? ptr_a : ptr_b;
      double *gv = other == 0 ? gs : gc;
      double s = 0.0, r = 0.0;
      for (int64_t j = ptr_c[p]; j < ptr_c[p + 1]; ++j) {
        const double *pj = pc + j * D;
        double r2 = 0.0;
        for (int d = 0; d < D; ++d) {
          const double t = pi[d] - pj[d];
          r2 += t * t;
        }
        const double wk = wc[j] * exp(-r2 * inv2s2);
        s += wk;
        r += wk * r2;
        for (int d = 0; d < nd; ++d) gv[d] += wk * (pi[dc + d] - pj[dc + d]);
      }
      if (dc == 0) {
        if (other == 0) {
          ss = s;
          rs = r;
        } else {
          sc = s;
          rc = r;
        }
      }
    }
    if (gout != nullptr)
      for (int d = 0; d < nd; ++d) gout[i * D + dc + d] = -s2 * w * gs[d] + s2 * w * gc[d];
  }
  if (wout != nullptr) wout[i] = 2.0 * ss - 2.0 * sc;
  double *rec = A.work + g * 4;
  rec[0] = w * ss;
  rec[1] = w * sc;
  rec[2] = w * rs;
  rec[3] = w * rc;
}

// One CTA per pair: Kxx, Kyy, Kxy and dL/dsigma from the per-point records,
// summed in a fixed order.
__global__ void __launch_bounds__(256) exact_pairs_kernel(ExactArgs A, double *Kxx, double *Kyy,
                                                          double *Kxy, double *loss,
                                                          double *grad_sigma) {
  __shared__ double sh[(256 / 32) * 5];
  const int64_t p = blockIdx.x;
  double v[5] = {0.0, 0.0, 0.0, 0.0, 0.0};  // w ss (x), w ss (y), w sc (x), rs+rs, rc (x)
  for (int64_t i = A.ptr_x[p] + threadIdx.x; i < A.ptr_x[p + 1]; i += blockDim.x) {
    const double *rec = A.work + i * 4;
    v[0] += rec[0];
    v[2] += rec[1];
    v[3] += rec[2];
    v[4] += rec[3];
  }
  for (int64_t j = A.ptr_y[p] + threadIdx.x; j < A.ptr_y[p + 1]; j += blockDim.x) {
    const double *rec = A.work + (A.NX + j) * 4;
    v[1] += rec[0];
    v[3] += rec[2];
  }
  block_sum_n<5>(v, sh);
  if (threadIdx.x == 0) {
    Kxx[p] = v[0];
    Kyy[p] = v[1];
    Kxy[p] = v[2];
    if (loss != nullptr) loss[p] = v[0] + v[1] - 2.0 * v[2];
    if (grad_sigma != nullptr) {
      const double s3 = A.sigma * A.sigma * A.sigma;
      grad_sigma[p] = (v[3] - 2.0 * v[4]) / s3;
    }
  }
}

// Dense matrices of one pair: G[i][j] = exp(-|a_i - b_j|^2 / (2 sigma^2)),
// diff[i][j][d] = a_i[d] - b_j[d] (kde_gradients.py:32-36).
__global__ void exact_matrices_kernel(const double *a, int64_t n, const double *b, int64_t m,
                                      int D, double sigma, double *G, double *diff) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= n * m) return;
  const int64_t i = t / m, j = t % m;
  double r2 = 0.0;
  for (int d = 0; d < D; ++d) {
    const double v = a[i * D + d] - b[j * D + d];
    r2 += v * v;
    if (diff != nullptr) diff[t * D + d] = v;
  }
  if (G != nullptr) G[t] = exp(-r2 / (2.0 * sigma * sigma));
}

}  // namespace ra
