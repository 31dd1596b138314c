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

#include "ra_chunks.cuh"
#include "ra_common.cuh"
#include "ra_prep.cuh"

namespace ra {

struct FinalizeArgs {
  int64_t P;
  const int64_t *item_off;
  const int64_t *boff;
  const double *itemK, *itemS;
  double *K_out[3];  // caller's Kxx, Kyy, Kxy ([P] each)
  double *K_ws;   // [3P] copy kept in the workspace
  double *S_ws;   // [3P]
  int *state;     // set to 1 when not null
};

// Pairs with at most kWarpItems work items are summed by one warp each
// (finalize_warp_kernel), larger ones by one CTA each (finalize_kernel).
constexpr int64_t kWarpItems = 256;

// The item range [base, end) of pair p: item_off[P] is the (clamped) number
// of items actually emitted, so partials beyond it are never read, even for
// a malformed ptr that overflowed the bound.
__device__ __forceinline__ void pair_items(const FinalizeArgs &A, int64_t p, int64_t &base,
                                           int64_t &end) {
  const int64_t lim = A.item_off[A.P];
  base = A.item_off[p];
  end = A.item_off[p + 1] < lim ? A.item_off[p + 1] : lim;
  if (base > end) base = end;
}

// One warp per pair of at most kWarpItems items (lane-strided sums, then a
// fixed shuffle tree: deterministic).  Block b of the items maps to K index
// (xy -> 2, xx -> 0, yy -> 1).
__global__ void __launch_bounds__(256) finalize_warp_kernel(FinalizeArgs A) {
  const int64_t p = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (p >= A.P) return;
  if (p == 0 && lane == 0 && A.state != nullptr) *A.state = 1;
  int64_t base, end;
  pair_items(A, p, base, end);
  if (end - base > kWarpItems) return;  // finalize_kernel
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
      A.K_out[kidx[b]][p] = k;
      A.K_ws[kidx[b] * A.P + p] = k;
      A.S_ws[kidx[b] * A.P + p] = s;
    }
  }
}

// One CTA per pair of more than kWarpItems items.  Four independent
// accumulators per thread keep enough loads in flight for pairs with hundreds
// of thousands of items.
template <int NT>
__global__ void __launch_bounds__(NT) finalize_kernel(FinalizeArgs A) {
  __shared__ double sh[NT / 32];
  for (int64_t p = blockIdx.x; p < A.P; p += gridDim.x) {
    int64_t base, end;
    pair_items(A, p, base, end);
    if (end - base <= kWarpItems) continue;  // finalize_warp_kernel
    const int kidx[3] = {2, 0, 1};
#pragma unroll 1
    for (int b = 0; b < 3; ++b) {
      int64_t b0 = base + A.boff[p * 4 + b];
      const int64_t b1 = b < 2 ? base + A.boff[p * 4 + b + 1] : base + A.boff[p * 4 + 3];
      const int64_t e = b1 < end ? b1 : end;
      if (b0 > e) b0 = e;
      double k[4] = {0.0, 0.0, 0.0, 0.0}, s[4] = {0.0, 0.0, 0.0, 0.0};
      int64_t i = b0 + threadIdx.x;
      for (; i + 3 * NT < e; i += 4 * NT) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          k[u] += A.itemK[i + u * NT];
          s[u] += A.itemS[i + u * NT];
        }
      }
      for (; i < e; i += NT) {
        k[0] += A.itemK[i];
        s[0] += A.itemS[i];
      }
      const double kt = block_sum((k[0] + k[1]) + (k[2] + k[3]), sh);
      const double st = block_sum((s[0] + s[1]) + (s[2] + s[3]), sh);
      if (threadIdx.x == 0) {
        A.K_out[kidx[b]][p] = kt;
        A.K_ws[kidx[b] * A.P + p] = kt;
        A.S_ws[kidx[b] * A.P + p] = st;
      }
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
  const int64_t *choff, *chx;  // chunk map (ra_chunks.cuh)
  const int32_t *cpair;
  unsigned *ticket;            // chunk counter of the launch, zeroed
  unsigned *pair_ticket;       // pair counter of epi3_small_kernel, zeroed
  double *rec;         // per-chunk (Q, R[DP]) partials, stride stats_stride(DP)
  const float *x, *y;  // original coordinates
  const uint8_t *mask_x, *mask_y;
  const ulonglong2 *tiles_x, *tiles_y;  // packed3: tile layout (ra_prep.cuh)
  const float *aw_x, *aw_y;             // packed3: a~ = a / m per slot
  const double *sigma_p;                // [P] per-pair bandwidths, or null
  const int64_t *tbase_x, *tbase_y;     // packed3: first tile of each pair
  int nq;                               // packed3: arrays per tile
  const float *Gx, *Gy, *Ax, *Ay;       // generic
  const float *accX, *accY;  // packed3: [tiles * 64][8]; generic: [num][acc_stride]
  int acc_stride;
  float *grad_x, *grad_y;
  double *grad_wx, *grad_wy;
  double *grad_sigma;
  int totals;  // the side totals R, Q are used (centering, or a weight gradient)
  int vec4;    // D % 4 == 0, grad_x, grad_y (and x, y when xraw) 16-byte aligned
  int xraw;    // no Gx / Gy (tensor-core layout): x' = c (x - anchor) from the points
  int *err;    // the workspace's error word (bounded waits of the ring passes)
};

// The packed coordinate x'_d of point g: stored (Gx / Gy), or recomputed from
// the caller's points exactly as the tensor-core packing pass computes it
// (x' = c ((x - hi) - lo) in fp32 from the anchor's fp32 pair), for the
// layout that stores only fp16 tiles.
__device__ __forceinline__ float packed_coord(const EpilogueArgs &A, int side, int64_t g, int d,
                                              const float *anc, float sc) {
  if (!A.xraw) return (side == 0 ? A.Gx : A.Gy)[g * A.DP + d];
  if (d >= A.D) return 0.f;
  return sc * (((side == 0 ? A.x : A.y)[g * A.D + d] - anc[d]) - anc[A.DP + d]);
}
// the anchor pairs (hi [DP], then lo [DP]) of a side, tensor-core layout
__device__ __forceinline__ const float *side_anchor(const EpilogueArgs &A, int64_t p, int side) {
  return tc_anchor(A.meta + p * meta_stride(A.DP), A.DP, side);
}
__device__ __forceinline__ float side_scale(const EpilogueArgs &A, int64_t p) {
  return A.sigma_p != nullptr ? scale_of_sigma(A.sigma_p[p]) : (float)A.scale;
}

// One point's record (self (s, G0..G2), cross (s, G0..G2), 32-byte aligned)
// and packed weight, loaded ahead of point_grads.
struct PointRec3 {
  float4 self4, cross4;
  float aw;
};
__device__ __forceinline__ PointRec3 load_point3(const EpilogueArgs &A, int side, int64_t slot) {
  static_assert(kAcc3Stride == 8 && kAcc3Block == 4, "record = two float4 blocks");
  const float4 *rec = reinterpret_cast<const float4 *>((side == 0 ? A.accX : A.accY) +
                                                       slot * kAcc3Stride);
  PointRec3 r;
  r.self4 = rec[0];
  r.cross4 = rec[1];
  r.aw = (side == 0 ? A.aw_x : A.aw_y)[slot];
  return r;
}

// Per-point backward quantities of the D <= 3 layout: `slot` = tile * 64 +
// lane of the point in the tile layout.  Returns gxt[0..D) (dL/dx~) and ga
// (dL/da, direct part).
// The tile kernel's sums carry the factor 1 / m of the cloud the point was
// paired with (m_own for the self block, m_par for the cross block), and the
// packed weight is a / m_own: both are undone here.
template <int MAXD>
__device__ __forceinline__ void point_grads(const PointRec3 &R, int D, double cs, double cc,
                                            double k_x, double m_own, double m_par, double *gxt,
                                            double &ga, double &a_out) {
  const float gs[3] = {R.self4.y, R.self4.z, R.self4.w};
  const float gc[3] = {R.cross4.y, R.cross4.z, R.cross4.w};
  const double a = (double)R.aw * m_own;
  const double ws = cs * m_own, wc = cc * m_par;
#pragma unroll
  for (int d = 0; d < MAXD; ++d) {
    // difference form: G = sum w k (x' - y') accumulated directly
    gxt[d] = d < D ? -a * k_x * (ws * gs[d] + wc * gc[d]) : 0.0;
  }
  ga = ws * R.self4.x + wc * R.cross4.x;
  a_out = a;
}

// Per (pair, side) constants of the epilogue.
struct EpiSide {
  double cxx, cyy, cxy, cs, cc, k_x, W, Wraw;
  double m_own, m_par;  // D <= 3: weight scales of this side and of the other
  const double *mu;
  int64_t s, span, count;
};

__device__ __forceinline__ EpiSide epi_side(const EpilogueArgs &A, int64_t p, int side) {
  EpiSide E;
  const Seg sg = A.seg[p];
  E.s = side == 0 ? sg.xs : sg.ys;
  E.span = side == 0 ? sg.xspan : sg.yspan;
  E.count = side == 0 ? sg.xcount : sg.ycount;
  E.cxx = A.coef[p];
  E.cyy = A.coef[A.P + p];
  E.cxy = A.coef[2 * A.P + p];
  E.cs = side == 0 ? 2.0 * E.cxx : 2.0 * E.cyy;
  E.cc = E.cxy;
  const double sgm = A.sigma_p != nullptr ? A.sigma_p[p] : A.sigma;
  const double sc = A.sigma_p != nullptr ? (double)scale_of_sigma(sgm) : A.scale;
  E.k_x = 1.0 / (sc * sgm * sgm);
  const double *meta = A.meta + p * meta_stride(A.DP);
  E.W = meta[side];
  E.Wraw = meta[2 + side];
  E.m_own = meta[meta_wscale(A.DP) + side];
  E.m_par = meta[meta_wscale(A.DP) + 1 - side];
  E.mu = meta + 4 + side * A.DP;
  return E;
}

// dL/dsigma per pair (every pair, empty ones included).
__global__ void sigma_grad_kernel(EpilogueArgs A) {
  const int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (p >= A.P) return;
  const double cxx = A.coef[p], cyy = A.coef[A.P + p], cxy = A.coef[2 * A.P + p];
  const double sg = A.sigma_p != nullptr ? A.sigma_p[p] : A.sigma;
  const double sc = A.sigma_p != nullptr ? (double)scale_of_sigma(sg) : A.scale;
  const double c2 = sc * sc, s3 = sg * sg * sg;
  const double Sxx = A.S_ws[p], Syy = A.S_ws[A.P + p], Sxy = A.S_ws[2 * A.P + p];
  A.grad_sigma[p] = (cxx * Sxx + cyy * Syy + cxy * Sxy) / (c2 * s3);
}

// dL/dw_i from dL/da_i (centering part already applied) -- kde.py weight
// normalisation: raw (identity), clamped sum, plain sum.
__device__ __forceinline__ double weight_grad(int wmode, double m, double gat, double Qt,
                                              const EpiSide &E) {
  if (wmode == 0) return m * gat;
  if (wmode == 2 && !(E.Wraw > 1e-8)) return m * gat / 1e-8;
  return m * (gat - Qt) / E.W;
}

// ---- D <= 3 (packed3): one thread per point --------------------------------
// The cloud-wide sums of one side that the Jacobians need, over points
// [b, e) of the side: R += dL/dx~_i (D values), Q += a_i dL/da_i.  The next
// point's record is in flight while this one is summed.
__device__ __forceinline__ void epi3_sum_points(const EpilogueArgs &A, const EpiSide &E, int side,
                                                int64_t slot0, int64_t b, int64_t e, int stride,
                                                double (&R)[3], double &Q) {
  PointRec3 cur;
  if (b < e) cur = load_point3(A, side, slot0 + b);
  for (int64_t i = b; i < e; i += stride) {
    PointRec3 nxt;
    if (i + stride < e) nxt = load_point3(A, side, slot0 + i + stride);
    double gxt[3], ga, a;
    point_grads<3>(cur, A.D, E.cs, E.cc, E.k_x, E.m_own, E.m_par, gxt, ga, a);
#pragma unroll
    for (int d = 0; d < 3; ++d) R[d] += gxt[d];  // gxt[d >= D] == 0
    Q += a * ga;
    cur = nxt;
  }
}

// Gradients of points [b, e) of one side (zeros for the padded tail of a
// dense row, i >= count), given the side's totals R and Qt = Q - mu . R.
__device__ __forceinline__ void epi3_write_points(const EpilogueArgs &A, const EpiSide &E,
                                                  int side, int64_t slot0, int64_t b, int64_t e,
                                                  int stride, const double (&R)[3], double Qt) {
  const int D = A.D;
  const float *pts = side == 0 ? A.x : A.y;
  const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
  const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
  float *gout = side == 0 ? A.grad_x : A.grad_y;
  double *wout = side == 0 ? A.grad_wx : A.grad_wy;
  // the next point's record is loaded before this point's stores (which
  // might alias it as far as the compiler knows)
  PointRec3 cur;
  if (b < e && b < E.count) cur = load_point3(A, side, slot0 + b);
  for (int64_t i = b; i < e; i += stride) {
    PointRec3 nxt;
    if (i + stride < e && i + stride < E.count) nxt = load_point3(A, side, slot0 + i + stride);
    const int64_t g = E.s + i;
    double gxt[3] = {0.0, 0.0, 0.0}, ga = 0.0, a = 0.0;
    const bool live = i < E.count;
    if (live) point_grads<3>(cur, D, E.cs, E.cc, E.k_x, E.m_own, E.m_par, gxt, ga, a);
    cur = nxt;
    if (gout != nullptr) {
#pragma unroll
      for (int d = 0; d < 3; ++d) {
        if (d >= D) break;
        double val = gxt[d];
        if (A.center && live) val -= a * R[d];
        gout[g * D + d] = (float)val;
      }
    }
    if (wout != nullptr && wmode != 3) {
      double gat = ga;
      if (A.center && live) {
#pragma unroll
        for (int d = 0; d < 3; ++d)
          if (d < D) gat -= (double)pts[g * D + d] * R[d];
      }
      const double m = (mask == nullptr || mask[g] != 0) ? 1.0 : 0.0;
      wout[g] = live ? weight_grad(wmode, m, gat, Qt, E) : 0.0;
    }
  }
}

__device__ __forceinline__ double epi3_qt(const EpilogueArgs &A, const EpiSide &E, double Q,
                                          const double (&R)[3]) {
  double Qt = Q;
  if (A.center) {
#pragma unroll
    for (int d = 0; d < 3; ++d)
      if (d < A.D) Qt -= E.mu[d] * R[d];
  }
  return Qt;
}

// ---- D <= 3, pairs with more than kSmallPts points on a side: two chunked
// passes, so that one pair spreads over many CTAs.
// Pass 1: per chunk, R = sum dL/dx~ (D values) and Q = sum a dL/da.
template <int NT>
__global__ void __launch_bounds__(NT) epi3_partial_kernel(EpilogueArgs A) {
  __shared__ double sh[(NT / 32) * 4];
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
  const int rs = stats_stride(A.DP);
  for_each_chunk(M, [&](int64_t p, int side, int64_t c, int64_t v, int64_t, int64_t) {
    if (small_pair(A.seg[p])) return;  // epi3_small_kernel
    const EpiSide E = epi_side(A, p, side);
    const int64_t slot0 = (side == 0 ? A.tbase_x : A.tbase_y)[p] * kTile;
    const int64_t b = c * kChunk, e = b + kChunk < E.count ? b + kChunk : E.count;
    double R[3] = {0.0, 0.0, 0.0}, Q = 0.0;
    epi3_sum_points(A, E, side, slot0, b + threadIdx.x, e, NT, R, Q);
    double *rec = A.rec + v * rs;
    double vals[4] = {Q, R[0], R[1], R[2]};
    block_sum_n<4>(vals, sh);
    if (threadIdx.x == 0) {
#pragma unroll
      for (int k = 0; k < 4; ++k) rec[k] = vals[k];
    }
  });
}

// Pass 2: per chunk, combine the side's partials (thread-strided over the
// chunks, fixed-order block sums) and write the gradients of the chunk's points.
template <int NT>
__global__ void __launch_bounds__(NT, 3) epi3_write_kernel(EpilogueArgs A) {
  __shared__ double sh[(NT / 32) * 4];
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
  const int rs = stats_stride(A.DP);
  for_each_chunk(M, [&](int64_t p, int side, int64_t c, int64_t, int64_t first, int64_t n) {
    if (small_pair(A.seg[p])) return;  // epi3_small_kernel
    const EpiSide E = epi_side(A, p, side);
    double R[3] = {0.0, 0.0, 0.0}, Q = 0.0;
    for (int64_t k = threadIdx.x; k < n; k += NT) {
      const double *r = A.rec + (first + k) * rs;
      Q += r[0];
      R[0] += r[1];
      R[1] += r[2];
      R[2] += r[3];
    }
    double vals[4] = {Q, R[0], R[1], R[2]};
    block_sum_n<4>(vals, sh);
    Q = vals[0];
#pragma unroll
    for (int d = 0; d < 3; ++d) R[d] = vals[1 + d];
    const int64_t slot0 = (side == 0 ? A.tbase_x : A.tbase_y)[p] * kTile;
    const int64_t b = c * kChunk, e = b + kChunk < E.span ? b + kChunk : E.span;
    epi3_write_points(A, E, side, slot0, b + threadIdx.x, e, NT, R, epi3_qt(A, E, Q, R));
  });
}

// ---- D <= 3, pairs with at most kSmallPts points per side (small_pair): one
// CTA per pair and side sums R and Q over the side's points, then writes
// their gradients (the records are re-read from cache), in one launch.
template <int NT>
__global__ void __launch_bounds__(NT, 3) epi3_small_kernel(EpilogueArgs A) {
  __shared__ double sh[(NT / 32) * 4];
  __shared__ unsigned pt_slot[2];
  unsigned pt_nxt = 0;
  int pt_k = 0;
  for (int64_t p = pair_ticket_first(A.pair_ticket, pt_slot); p < A.P;
       p = pair_ticket_next(pt_slot, ++pt_k, pt_nxt)) {
    pt_nxt = pair_ticket_take(A.pair_ticket);
    if (!small_pair(A.seg[p])) continue;
    for (int side = 0; side < 2; ++side) {
      const EpiSide E = epi_side(A, p, side);
      const int64_t slot0 = (side == 0 ? A.tbase_x : A.tbase_y)[p] * kTile;
      double R[3] = {0.0, 0.0, 0.0}, Q = 0.0;
      epi3_sum_points(A, E, side, slot0, threadIdx.x, E.count, NT, R, Q);
      double vals[4] = {Q, R[0], R[1], R[2]};
      block_sum_n<4>(vals, sh);
      Q = vals[0];
#pragma unroll
      for (int d = 0; d < 3; ++d) R[d] = vals[1 + d];
      epi3_write_points(A, E, side, slot0, threadIdx.x, E.span, NT, R, epi3_qt(A, E, Q, R));
    }
  }
}

// ---- generic D: RW = DP threads per point (one per dimension) -------------
__device__ __forceinline__ double gen_gxt(const EpilogueArgs &A, int side, int64_t g, int d,
                                          const EpiSide &E, double &a, double &ga) {
  const int DP = A.DP;
  const float *acc = (side == 0 ? A.accX : A.accY) + g * A.acc_stride;
  a = (side == 0 ? A.Ax : A.Ay)[g];
  // the stored self sums leave out the diagonal term (k_ii = 1, weight a_i)
  const double s_self = acc[2 * DP], s_cross = acc[2 * DP + 1];
  ga = E.cs * (s_self + a) + E.cc * s_cross;
  if (d >= A.D) return 0.0;
  const double xp = (side == 0 ? A.Gx : A.Gy)[g * DP + d];
  const double Gs = xp * s_self - (double)acc[d];
  const double Gc = xp * s_cross - (double)acc[DP + d];
  return -a * E.k_x * (E.cs * Gs + E.cc * Gc);
}

template <int NT>
__global__ void __launch_bounds__(NT) epig_partial_kernel(EpilogueArgs A) {
  __shared__ double sh[NT];
  __shared__ double shd[NT];
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
  const int DP = A.DP, RW = DP;  // generic DP is a power of two >= 4 and <= NT
  const int lanes = NT / RW;
  const int tid = threadIdx.x, d = tid % RW, pl = tid / RW;
  const int rs = stats_stride(DP);
  for_each_chunk(M, [&](int64_t p, int side, int64_t c, int64_t v, int64_t, int64_t) {
    const EpiSide E = epi_side(A, p, side);
    const int64_t b = c * kChunk, e = b + kChunk < E.count ? b + kChunk : E.count;
    double Rd = 0.0, Q = 0.0;
    for (int64_t i = b + pl; i < e; i += lanes) {
      double a, ga;
      Rd += gen_gxt(A, side, E.s + i, d, E, a, ga);
      if (d == 0) Q += a * ga;
    }
    sh[tid] = Rd;
    shd[tid] = Q;
    __syncthreads();
    double *rec = A.rec + v * rs;
    if (tid < DP) {
      double t = 0.0;
      for (int l = 0; l < lanes; ++l) t += sh[l * RW + tid];
      rec[1 + tid] = t;
    }
    if (tid == 0) {
      double t = 0.0;
      for (int l = 0; l < lanes; ++l) t += shd[l * RW];
      rec[0] = t;
    }
    __syncthreads();
  });
}

template <int NT>
__global__ void __launch_bounds__(NT) epig_write_kernel(EpilogueArgs A) {
  __shared__ double sh[NT];
  __shared__ double shd[NT];
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
  const int D = A.D, DP = A.DP, RW = DP;
  const int lanes = NT / RW;
  const int tid = threadIdx.x, d = tid % RW, pl = tid / RW;
  const int rs = stats_stride(DP);
  for_each_chunk(M, [&](int64_t p, int side, int64_t c, int64_t, int64_t first, int64_t n) {
    const EpiSide E = epi_side(A, p, side);
    // totals of the side: point lane pl takes chunks pl, pl + lanes, ...
    double Rd = 0.0, Q = 0.0;
    for (int64_t k = pl; k < n; k += lanes) {
      const double *r = A.rec + (first + k) * rs;
      Rd += r[1 + d];
      if (d == 0) Q += r[0];
    }
    sh[tid] = Rd;
    shd[tid] = Q;
    __syncthreads();
    double Rtot = 0.0, Qtot = 0.0;
    for (int l = 0; l < lanes; ++l) Rtot += sh[l * RW + d];
    for (int l = 0; l < lanes; ++l) Qtot += shd[l * RW];
    __syncthreads();
    // mu . R
    sh[tid] = (pl == 0 && d < D) ? E.mu[d] * Rtot : 0.0;
    __syncthreads();
    double muR = 0.0;
    for (int k = 0; k < RW; ++k) muR += sh[k];
    __syncthreads();
    const double Qt = A.center ? Qtot - muR : Qtot;

    const float *pts = side == 0 ? A.x : A.y;
    const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
    const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
    float *gout = side == 0 ? A.grad_x : A.grad_y;
    double *wout = side == 0 ? A.grad_wx : A.grad_wy;
    const int64_t b = c * kChunk, e = b + kChunk < E.span ? b + kChunk : E.span;
    for (int64_t i0 = b; i0 < e; i0 += lanes) {
      const int64_t i = i0 + pl;
      const bool inb = i < e;
      const bool live = i < E.count && inb;
      const int64_t g = E.s + i;
      double a = 0.0, ga = 0.0, gx = 0.0;
      if (live) gx = gen_gxt(A, side, g, d, E, a, ga);
      if (A.center && live) gx -= a * Rtot;
      if (inb && gout != nullptr && d < D) gout[g * D + d] = (float)gx;
      // x_i . R across the RW threads of this point
      sh[tid] = (live && d < D && A.center) ? (double)pts[g * D + d] * Rtot : 0.0;
      __syncthreads();
      if (d == 0 && inb && wout != nullptr && wmode != 3) {
        double xr = 0.0;
        for (int k = 0; k < RW; ++k) xr += sh[pl * RW + k];
        const double m = (mask == nullptr || mask[g] != 0) ? 1.0 : 0.0;
        wout[g] = live ? weight_grad(wmode, m, ga - xr, Qt, E) : 0.0;
      }
      __syncthreads();
    }
  });
}

// ---- generic D, wide points (DP >= 32): one warp per point ----------------
// Lane l handles coordinates l, l + 32, ...; chunk partials are combined over
// the 8 warps in order (deterministic), the dot products x . R by warp
// shuffles -- no barrier per point.
__device__ __forceinline__ double genw_gxt(const EpilogueArgs &A, const float *acc, double a,
                                           double s_self, double s_cross, double xp,
                                           int d, const EpiSide &E) {
  const int DP = A.DP;
  const double Gs = xp * s_self - (double)acc[d];
  const double Gc = xp * s_cross - (double)acc[DP + d];
  return -a * E.k_x * (E.cs * Gs + E.cc * Gc);
}

template <int DP>
__global__ void __launch_bounds__(256) epigw_partial_kernel(EpilogueArgs A) {
  constexpr int NW = 8, KL = DP / 32;
  __shared__ double sh[NW][DP + 1];
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int D = A.D, rs = stats_stride(DP);
  for_each_chunk(M, [&](int64_t p, int side, int64_t c, int64_t v, int64_t, int64_t) {
    const EpiSide E = epi_side(A, p, side);
    const float *accb = side == 0 ? A.accX : A.accY;
    const float *Ap = side == 0 ? A.Ax : A.Ay;
    const float *anc = side_anchor(A, p, side);
    const float scl = side_scale(A, p);
    const int64_t b = c * kChunk, e = b + kChunk < E.count ? b + kChunk : E.count;
    double R[KL], Q = 0.0;
#pragma unroll
    for (int k = 0; k < KL; ++k) R[k] = 0.0;
    // software-pipelined: the next point's loads are in flight while this
    // one is summed (same points, same order)
    struct Pt {
      float a, ss, sc, ts[KL], tc[KL], xp[KL];
    };
    auto load = [&](int64_t i) {
      Pt q;
      const int64_t g = E.s + i;
      const float *acc = accb + g * A.acc_stride;
      q.a = Ap[g];
      q.ss = acc[2 * DP];
      q.sc = acc[2 * DP + 1];
#pragma unroll
      for (int k = 0; k < KL; ++k) {
        const int d = lane + 32 * k;
        q.ts[k] = d < D ? acc[d] : 0.f;
        q.tc[k] = d < D ? acc[DP + d] : 0.f;
        q.xp[k] = d < D ? packed_coord(A, side, g, d, anc, scl) : 0.f;
      }
      return q;
    };
    Pt cur;
    if (b + wid < e) cur = load(b + wid);
    for (int64_t i = b + wid; i < e; i += NW) {
      Pt nxt;
      if (i + NW < e) nxt = load(i + NW);
      const double a = cur.a, s_self = cur.ss, s_cross = cur.sc;
#pragma unroll
      for (int k = 0; k < KL; ++k) {
        if (lane + 32 * k < D) {
          const double xp = cur.xp[k];
          const double Gs = xp * s_self - (double)cur.ts[k];
          const double Gc = xp * s_cross - (double)cur.tc[k];
          R[k] += -a * E.k_x * (E.cs * Gs + E.cc * Gc);
        }
      }
      // the stored self sums leave out the diagonal term (k_ii = 1, weight a_i)
      Q += a * (E.cs * (s_self + a) + E.cc * s_cross);
      cur = nxt;
    }
#pragma unroll
    for (int k = 0; k < KL; ++k) sh[wid][lane + 32 * k] = R[k];
    if (lane == 0) sh[wid][DP] = Q;
    __syncthreads();
    double *rec = A.rec + v * rs;
    for (int t = tid; t < DP + 1; t += 256) {
      double tot = 0.0;
      for (int q = 0; q < NW; ++q) tot += sh[q][t];
      if (t < DP) rec[1 + t] = tot;
      else rec[0] = tot;
    }
    __syncthreads();
  });
}

template <int DP>
__global__ void __launch_bounds__(256) epigw_write_kernel(EpilogueArgs A) {
  constexpr int NW = 8, KL = DP / 32;
  __shared__ double Rsh[DP + 1];
  __shared__ double red[NW];
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int D = A.D, rs = stats_stride(DP);
  for_each_chunk(M, [&](int64_t p, int side, int64_t c, int64_t, int64_t first, int64_t n) {
    const EpiSide E = epi_side(A, p, side);
    // the side's totals, summed over its chunks in order (zero when no
    // output uses them: the partial pass did not run)
    for (int t = tid; t < DP + 1; t += 256) {
      double tot = 0.0;
      if (A.totals)
        for (int64_t kk = 0; kk < n; ++kk) tot += A.rec[(first + kk) * rs + (t < DP ? 1 + t : 0)];
      Rsh[t] = tot;  // Rsh[DP] = Q
    }
    __syncthreads();
    double mr = 0.0;
    for (int t = tid; t < D; t += 256) mr += E.mu[t] * Rsh[t];
    mr = warp_sum(mr);
    if (lane == 0) red[wid] = mr;
    __syncthreads();
    double muR = 0.0;
    for (int q = 0; q < NW; ++q) muR += red[q];
    const double Qt = A.center ? Rsh[DP] - muR : Rsh[DP];

    const float *pts = side == 0 ? A.x : A.y;
    const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
    const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
    float *gout = side == 0 ? A.grad_x : A.grad_y;
    double *wout = side == 0 ? A.grad_wx : A.grad_wy;
    const float *accb = side == 0 ? A.accX : A.accY;
    const float *Gp = side == 0 ? A.Gx : A.Gy;
    const float *Ap = side == 0 ? A.Ax : A.Ay;
    const float *anc = side_anchor(A, p, side);
    const float scl = side_scale(A, p);
    const int64_t b = c * kChunk, e = b + kChunk < E.span ? b + kChunk : E.span;

    // weight gradients: a warp per point, 4 points in flight, x . R by shuffles
    if (wout != nullptr && wmode != 3) {
      for (int64_t i0 = b + 4 * wid; i0 < e; i0 += 4 * NW) {
        double xr[4] = {0.0, 0.0, 0.0, 0.0};
        if (A.center) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int64_t i = i0 + u;
            if (i < e && i < E.count) {
              const int64_t g = E.s + i;
#pragma unroll
              for (int k = 0; k < KL; ++k) {
                const int dd = lane + 32 * k;
                if (dd < D) xr[u] += (double)pts[g * D + dd] * Rsh[dd];
              }
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) xr[u] = warp_sum(xr[u]);
        if (lane < 4) {
          const int64_t i = i0 + lane;
          if (i < e) {
            const int64_t g = E.s + i;
            double gw = 0.0;
            if (i < E.count) {
              const float *acc = accb + g * A.acc_stride;
              const double a = Ap[g], s_self = acc[2 * DP], s_cross = acc[2 * DP + 1];
              const double ga = E.cs * (s_self + a) + E.cc * s_cross;
              const double m = (mask == nullptr || mask[g] != 0) ? 1.0 : 0.0;
              const double xrl = lane == 0 ? xr[0] : lane == 1 ? xr[1] : lane == 2 ? xr[2] : xr[3];
              gw = weight_grad(wmode, m, ga - xrl, Qt, E);
            }
            wout[g] = gw;
          }
        }
      }
    }
    // position gradients over flat elements: float4 (point, 4 coordinates)
    // when D is a multiple of 4 -- a thread then keeps one coordinate chunk
    // and loads each point's scalars once per 4 coordinates -- else scalars
    if (gout != nullptr && A.vec4) {
      constexpr int NC = DP / 4;
      const int ncd = D / 4;  // chunks that hold coordinates
      const int cc = tid % NC;
      // this thread's anchor pairs (its coordinate chunk is fixed)
      const bool cl = A.xraw && cc < ncd;
      const float ah0 = cl ? anc[4 * cc] : 0.f, ah1 = cl ? anc[4 * cc + 1] : 0.f;
      const float ah2 = cl ? anc[4 * cc + 2] : 0.f, ah3 = cl ? anc[4 * cc + 3] : 0.f;
      const float al0 = cl ? anc[DP + 4 * cc] : 0.f, al1 = cl ? anc[DP + 4 * cc + 1] : 0.f;
      const float al2 = cl ? anc[DP + 4 * cc + 2] : 0.f, al3 = cl ? anc[DP + 4 * cc + 3] : 0.f;
      const int64_t nel = (e - b) * NC;
      constexpr int kAhead = 2;  // 4 doubles the registers (126 -> 156) for nothing
      for (int64_t k0 = tid; k0 < nel; k0 += kAhead * 256) {
        // the loads of kAhead elements go out before the first store (a
        // store to gout might alias them as far as the compiler knows)
        float4 ts[kAhead], tc[kAhead], xp[kAhead];
        float av[kAhead], ssv[kAhead], scv[kAhead];
#pragma unroll
        for (int u = 0; u < kAhead; ++u) {
          const int64_t k = k0 + u * 256;
          const int64_t i = b + k / NC;
          if (k < nel && cc < ncd && i < E.count) {
            const int64_t g = E.s + i;
            const float *acc = accb + g * A.acc_stride;
            av[u] = Ap[g];
            ssv[u] = acc[2 * DP];
            scv[u] = acc[2 * DP + 1];
            ts[u] = *reinterpret_cast<const float4 *>(acc + 4 * cc);
            tc[u] = *reinterpret_cast<const float4 *>(acc + DP + 4 * cc);
            if (A.xraw) {
              // the points themselves (16-byte aligned: vec4), packed here
              const float4 r = *reinterpret_cast<const float4 *>(pts + g * D + 4 * cc);
              xp[u] = make_float4(scl * ((r.x - ah0) - al0), scl * ((r.y - ah1) - al1),
                                  scl * ((r.z - ah2) - al2), scl * ((r.w - ah3) - al3));
            } else {
              xp[u] = *reinterpret_cast<const float4 *>(Gp + g * DP + 4 * cc);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < kAhead; ++u) {
          const int64_t k = k0 + u * 256;
          if (k < nel && cc < ncd) {
            const int64_t i = b + k / NC;
            const int64_t g = E.s + i;
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < E.count) {
              const double a = av[u], s_self = ssv[u], s_cross = scv[u];
              const float tsv[4] = {ts[u].x, ts[u].y, ts[u].z, ts[u].w};
              const float tcv[4] = {tc[u].x, tc[u].y, tc[u].z, tc[u].w};
              const float xv[4] = {xp[u].x, xp[u].y, xp[u].z, xp[u].w};
              float r[4];
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                const double Gs = xv[v] * s_self - (double)tsv[v];
                const double Gc = xv[v] * s_cross - (double)tcv[v];
                double gx = -a * E.k_x * (E.cs * Gs + E.cc * Gc);
                if (A.center) gx -= a * Rsh[4 * cc + v];
                r[v] = (float)gx;
              }
              o = make_float4(r[0], r[1], r[2], r[3]);
            }
            *reinterpret_cast<float4 *>(gout + g * D + 4 * cc) = o;
          }
        }
      }
    } else if (gout != nullptr) {
      const int64_t nel = (e - b) * D;
      for (int64_t k0 = tid; k0 < nel; k0 += 4 * 256) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t k = k0 + u * 256;
          if (k < nel) {
            const int64_t i = b + k / D;
            const int dd = (int)(k % D);
            const int64_t g = E.s + i;
            double gx = 0.0;
            if (i < E.count) {
              const float *acc = accb + g * A.acc_stride;
              const double a = Ap[g];
              gx = genw_gxt(A, acc, a, acc[2 * DP], acc[2 * DP + 1],
                            (double)packed_coord(A, side, g, dd, anc, scl), dd, E);
              if (A.center) gx -= a * Rsh[dd];
            }
            gout[g * D + dd] = (float)gx;
          }
        }
      }
    }
    __syncthreads();  // Rsh and red are rewritten by the next chunk
  });
}

}  // namespace ra
