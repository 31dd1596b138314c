// ra_epilogue.cuh -- per-pair finalisation of the K/S sums and the backward
// epilogue that turns the per-point row sums into gradients.
//
// Backward math (pre-scaled coordinates x' = c (x~ - anchor), c = sqrt(log2 e / (2 sigma^2))):
//   G'_i  = c * sum_j w_j k_ij (x~_i - y~_j), accumulated directly by the D <= 3
//           kernel and as x'_i s_i - T_i (T = sum w k y') by the generic one
//   dL/dx~_i = -(a_i / (c sigma^2)) (2 cxx G'_self,i + cxy G'_cross,i)
//   dL/da_i  = 2 cxx s_self,i + cxy s_cross,i                (kde_gradients.py:98-113)
// then the centering Jacobian of x~ = x - sum_k a_k x_k (kde.py:77-81, 202-208):
//   dL/dx_i  = dL/dx~_i - a_i R,   R = sum_k dL/dx~_k
//   dL/da_i += -x_i . R
// and the weight normalisation a = w / W (kde.py:20-27, 115-121, 169-199):
//   dL/dw_i  = (dL/da_i - sum_k a_k dL/da_k) / W
// sigma: dK/dsigma = S / sigma^3 with S = sum w w' k r^2 (kde_gradients.py:115-123).
#pragma once

#include "ra_common.cuh"
#include "ra_prep.cuh"

namespace ra {

struct FinalizeArgs {
  int64_t P;
  const int64_t *item_off;
  const int64_t *boff;
  const double *itemK, *itemS;
  double *K_out;  // [3P] Kxx | Kyy | Kxy (caller's buffer)
  double *K_ws;   // [3P] copy kept in the workspace
  double *S_ws;   // [3P]
};

// one warp per pair; block b of the items maps to K index (xy -> 2, xx -> 0, yy -> 1)
__global__ void finalize_kernel(FinalizeArgs A) {
  const int64_t p = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (p >= A.P) return;
  // item_off[P] is the (clamped) number of items actually emitted: never read
  // partials beyond it, even for a malformed ptr that overflowed the bound
  const int64_t lim = A.item_off[A.P];
  const int64_t base = A.item_off[p];
  const int64_t end = A.item_off[p + 1] < lim ? A.item_off[p + 1] : lim;
  const int kidx[3] = {2, 0, 1};
#pragma unroll
  for (int b = 0; b < 3; ++b) {
    int64_t b0 = base + A.boff[p * 4 + b];
    const int64_t b1 = b < 2 ? base + A.boff[p * 4 + b + 1] : base + A.boff[p * 4 + 3];
    const int64_t e = b1 < end ? b1 : end;
    if (b0 > e) b0 = e;
    double k = 0.0, s = 0.0;
    for (int64_t i = b0 + lane; i < e; i += 32) {
      k += A.itemK[i];
      s += A.itemS[i];
    }
    k = warp_sum(k);
    s = warp_sum(s);
    if (lane == 0) {
      A.K_out[kidx[b] * A.P + p] = k;
      A.K_ws[kidx[b] * A.P + p] = k;
      A.S_ws[kidx[b] * A.P + p] = s;
    }
  }
}

struct EpilogueArgs {
  int64_t P;
  int D, DP;
  int packed3;
  int center;
  int wmode_x, wmode_y;
  double scale;      // c
  double sigma;
  const Seg *seg;
  const double *meta;
  const double *coef;  // [3P]: dL/dKxx | dL/dKyy | dL/dKxy
  const double *S_ws;  // [3P]
  const float *x, *y;  // original coordinates
  const uint8_t *mask_x, *mask_y;
  const ulonglong2 *tiles_x, *tiles_y;  // packed3: tile layout (ra_prep.cuh)
  const int64_t *tbase_x, *tbase_y;     // packed3: first tile of each pair
  int nq;                               // packed3: arrays per tile
  const float *Gx, *Gy, *Ax, *Ay;       // generic
  const float *accX, *accY;  // packed3: [tiles * 64][8]; generic: [num][acc_stride]
  int acc_stride;
  float *grad_x, *grad_y;
  double *grad_wx, *grad_wy;
  double *grad_sigma;
};

// Per-point backward quantities.  packed3: `slot` = tile * 64 + lane of the
// point in the tile layout; generic: `slot` = the point's row index.
// Returns gxt[0..D) (dL/dx~) and ga (dL/da, direct part).
template <int MAXD>
__device__ __forceinline__ void point_grads(const EpilogueArgs &A, int side, int64_t slot,
                                            double cs, double cc, double k_x, double *gxt,
                                            double &ga, double &a_out) {
  const int D = A.D;
  const float *acc = (side == 0 ? A.accX : A.accY) + slot * A.acc_stride;
  double a;
  double xp[MAXD];
  if (A.packed3) {
    const ulonglong2 *tiles = side == 0 ? A.tiles_x : A.tiles_y;
    const int64_t t = slot / kTile, l = slot % kTile;
    const ulonglong2 q0 = tiles[(t * A.nq) * kTile + l];
    const ulonglong2 q1 = tiles[(t * A.nq + 1) * kTile + l];
    xp[0] = lo_of(q0.x);
    if (MAXD > 1) xp[1] = lo_of(q0.y);
    if (MAXD > 2) xp[2] = lo_of(q1.x);
    a = lo_of(q1.y);
  } else {
    a = (side == 0 ? A.Ax : A.Ay)[slot];
    const float *gp = (side == 0 ? A.Gx : A.Gy) + slot * A.DP;
    for (int d = 0; d < D && d < MAXD; ++d) xp[d] = gp[d];
  }
  const int cross = A.packed3 ? kAcc3Block : 1 + A.DP;
  const double s_self = acc[0], s_cross = acc[cross];
  for (int d = 0; d < D && d < MAXD; ++d) {
    double Gs, Gc;
    if (A.packed3) {  // difference form: G = sum w k (x' - y') directly
      Gs = acc[1 + d];
      Gc = acc[cross + 1 + d];
    } else {          // folded form: G = x' s - sum w k y'
      Gs = xp[d] * s_self - (double)acc[1 + d];
      Gc = xp[d] * s_cross - (double)acc[cross + 1 + d];
    }
    gxt[d] = -a * k_x * (cs * Gs + cc * Gc);
  }
  ga = cs * s_self + cc * s_cross;
  a_out = a;
}

// One CTA per (pair, side), one thread per point; D <= 3 (packed3) only.
template <int NT>
__global__ void __launch_bounds__(NT) epilogue3_kernel(EpilogueArgs A) {
  __shared__ double sh[NT / 32];
  const int64_t p = blockIdx.x >> 1;
  const int side = blockIdx.x & 1;
  if (p >= A.P) return;
  const Seg sg = A.seg[p];
  const int64_t s = side == 0 ? sg.xs : sg.ys;
  const int64_t span = side == 0 ? sg.xspan : sg.yspan;
  const int64_t count = side == 0 ? sg.xcount : sg.ycount;
  const int D = A.D;
  const double cxx = A.coef[p], cyy = A.coef[A.P + p], cxy = A.coef[2 * A.P + p];
  const double cs = side == 0 ? 2.0 * cxx : 2.0 * cyy;
  const double cc = cxy;
  const double k_x = 1.0 / (A.scale * A.sigma * A.sigma);
  const double *meta = A.meta + p * meta_stride(A.DP);
  const double W = meta[side], Wraw = meta[2 + side];
  const double *mu = meta + 4 + side * A.DP;
  const float *pts = side == 0 ? A.x : A.y;
  const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
  const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
  float *gout = side == 0 ? A.grad_x : A.grad_y;
  double *wout = side == 0 ? A.grad_wx : A.grad_wy;

  const int64_t slot0 = (side == 0 ? A.tbase_x : A.tbase_y)[p] * kTile;
  // pass 1: R = sum dL/dx~ (D values), Q = sum a dL/da
  double R[3] = {0.0, 0.0, 0.0}, Q = 0.0;
  for (int64_t i = threadIdx.x; i < count; i += NT) {
    double gxt[3], ga, a;
    point_grads<3>(A, side, slot0 + i, cs, cc, k_x, gxt, ga, a);
    for (int d = 0; d < D; ++d) R[d] += gxt[d];
    Q += a * ga;
  }
  for (int d = 0; d < D; ++d) R[d] = block_sum(R[d], sh);
  Q = block_sum(Q, sh);
  double Qt = Q;
  if (A.center)
    for (int d = 0; d < D; ++d) Qt -= mu[d] * R[d];

  // pass 2: gradients (zeros for the padded tail of a dense row)
  for (int64_t i = threadIdx.x; i < span; i += NT) {
    const int64_t g = s + i;
    double gxt[3] = {0.0, 0.0, 0.0}, ga = 0.0, a = 0.0;
    const bool live = i < count;
    if (live) point_grads<3>(A, side, slot0 + i, cs, cc, k_x, gxt, ga, a);
    if (gout != nullptr) {
      for (int d = 0; d < D; ++d) {
        double v = gxt[d];
        if (A.center && live) v -= a * R[d];
        gout[g * D + d] = (float)v;
      }
    }
    if (wout != nullptr && wmode != 3) {
      double gat = ga;
      if (A.center && live)
        for (int d = 0; d < D; ++d) gat -= (double)pts[g * D + d] * R[d];
      const double m = (mask == nullptr || mask[g] != 0) ? 1.0 : 0.0;
      double gw;
      if (!live) {
        gw = 0.0;
      } else if (wmode == 0) {
        gw = m * gat;
      } else if (wmode == 2 && !(Wraw > 1e-8)) {
        gw = m * gat / 1e-8;
      } else {
        gw = m * (gat - Qt) / W;
      }
      wout[g] = gw;
    }
  }
  if (side == 0 && threadIdx.x == 0 && A.grad_sigma != nullptr) {
    const double c2 = A.scale * A.scale, s3 = A.sigma * A.sigma * A.sigma;
    const double Sxx = A.S_ws[p], Syy = A.S_ws[A.P + p], Sxy = A.S_ws[2 * A.P + p];
    A.grad_sigma[p] = (cxx * Sxx + cyy * Syy + cxy * Sxy) / (c2 * s3);
  }
}

// Generic D: one CTA per (pair, side); RW threads per point (one per dim).
template <int NT>
__global__ void __launch_bounds__(NT) epilogueg_kernel(EpilogueArgs A) {
  __shared__ double sh[NT];
  __shared__ double shd[NT];
  const int64_t p = blockIdx.x >> 1;
  const int side = blockIdx.x & 1;
  if (p >= A.P) return;
  const Seg sg = A.seg[p];
  const int64_t s = side == 0 ? sg.xs : sg.ys;
  const int64_t span = side == 0 ? sg.xspan : sg.yspan;
  const int64_t count = side == 0 ? sg.xcount : sg.ycount;
  const int D = A.D, DP = A.DP;
  const int RW = DP;  // generic DP is a power of two >= 4 and <= NT
  const int lanes = NT / RW;
  const int tid = threadIdx.x, d = tid % RW, pl = tid / RW;
  const double cxx = A.coef[p], cyy = A.coef[A.P + p], cxy = A.coef[2 * A.P + p];
  const double cs = side == 0 ? 2.0 * cxx : 2.0 * cyy;
  const double cc = cxy;
  const double k_x = 1.0 / (A.scale * A.sigma * A.sigma);
  const double *meta = A.meta + p * meta_stride(DP);
  const double W = meta[side], Wraw = meta[2 + side];
  const double *mu = meta + 4 + side * DP;
  const float *pts = side == 0 ? A.x : A.y;
  const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
  const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
  float *gout = side == 0 ? A.grad_x : A.grad_y;
  double *wout = side == 0 ? A.grad_wx : A.grad_wy;
  const float *accb = side == 0 ? A.accX : A.accY;
  const float *Gp = side == 0 ? A.Gx : A.Gy;
  const float *Ap = side == 0 ? A.Ax : A.Ay;
  const int cross = 1 + DP;

  auto gxt_of = [&](int64_t g, double &a, double &ga) -> double {
    const float *acc = accb + g * A.acc_stride;
    a = Ap[g];
    const double s_self = acc[0], s_cross = acc[cross];
    ga = cs * s_self + cc * s_cross;
    if (d >= D) return 0.0;
    const double xp = Gp[g * DP + d];
    const double Gs = xp * s_self - (double)acc[1 + d];
    const double Gc = xp * s_cross - (double)acc[cross + 1 + d];
    return -a * k_x * (cs * Gs + cc * Gc);
  };

  double Rd = 0.0, Q = 0.0;
  for (int64_t i = pl; i < count; i += lanes) {
    double a, ga;
    Rd += gxt_of(s + i, a, ga);
    if (d == 0) Q += a * ga;
  }
  sh[tid] = Rd;
  shd[tid] = Q;
  __syncthreads();
  double Rtot = 0.0;
  for (int l = 0; l < lanes; ++l) Rtot += sh[l * RW + d];
  double Qtot = 0.0;
  for (int l = 0; l < lanes; ++l) Qtot += shd[l * RW];
  __syncthreads();
  // mu . R
  sh[tid] = (pl == 0 && d < D) ? mu[d] * Rtot : 0.0;
  __syncthreads();
  double muR = 0.0;
  for (int e = 0; e < RW; ++e) muR += sh[e];
  __syncthreads();
  const double Qt = A.center ? Qtot - muR : Qtot;

  for (int64_t i0 = 0; i0 < span; i0 += lanes) {
    const int64_t i = i0 + pl;
    const bool inb = i < span;
    const bool live = i < count;
    const int64_t g = s + i;
    double a = 0.0, ga = 0.0, gx = 0.0;
    if (live) gx = gxt_of(g, a, ga);
    if (A.center && live) gx -= a * Rtot;
    if (inb && gout != nullptr && d < D) gout[g * D + d] = (float)gx;
    // x_i . R across the RW threads of this point
    sh[tid] = (live && d < D && A.center) ? (double)pts[g * D + d] * Rtot : 0.0;
    __syncthreads();
    if (d == 0 && inb && wout != nullptr && wmode != 3) {
      double xr = 0.0;
      for (int e = 0; e < RW; ++e) xr += sh[pl * RW + e];
      const double gat = ga - xr;
      const double m = (mask == nullptr || mask[g] != 0) ? 1.0 : 0.0;
      double gw;
      if (!live) gw = 0.0;
      else if (wmode == 0) gw = m * gat;
      else if (wmode == 2 && !(Wraw > 1e-8)) gw = m * gat / 1e-8;
      else gw = m * (gat - Qt) / W;
      wout[g] = gw;
    }
    __syncthreads();
  }
  if (side == 0 && tid == 0 && A.grad_sigma != nullptr) {
    const double c2 = A.scale * A.scale, s3 = A.sigma * A.sigma * A.sigma;
    const double Sxx = A.S_ws[p], Syy = A.S_ws[A.P + p], Sxy = A.S_ws[2 * A.P + p];
    A.grad_sigma[p] = (cxx * Sxx + cyy * Syy + cxy * Sxy) / (c2 * s3);
  }
}

}  // namespace ra
