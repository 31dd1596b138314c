// ra_prep.cuh -- per-pair preparation: segment bounds, weight normalisation,
// weighted centroids and packing of the points into the layouts the tile
// kernels read.
//
// Semantics follow rapidalign/kde.py:
//   ptr checks            kde.py:124-156 (plus a monotonicity check)
//   weight normalisation  kde.py:20-27 (single), 169-199 (ragged),
//                         115-121 (dense, clamped), 183-188 (uniform)
//   centering             kde.py:77-81, 202-208, 246-253
// Distances are translation invariant, so without centering both clouds are
// shifted by one common anchor (the unweighted mean of the x points); this
// keeps the packed coordinates small and changes no result.
//
// Pipeline: segment_kernel (bounds, ptr checks, chunk map) -> stats_kernel (per-chunk partial sums) -> meta_kernel (per pair, combines
// the partials in chunk order) -> pack kernels (per chunk).
#pragma once

#include "ra_chunks.cuh"
#include "ra_common.cuh"

namespace ra {

// Per-pair metadata (fp64), layout with DP = padded dimension:
//   [0] Wx  normaliser of x weights (a = w' / Wx; 1 for raw weights)
//   [1] Wy
//   [2] Wx_raw  sum of effective x weights before clamping
//   [3] Wy_raw
//   [4, 4+DP)        mu_x   (weighted centroid, sum_i a_i x_i)
//   [4+DP, 4+2DP)    mu_y
//   [4+2DP, 4+3DP)   anchor subtracted from x before packing
//   [4+3DP, 4+4DP)   anchor subtracted from y before packing
//   [4+4DP + side]   D <= 3 layout: the side's weight scale m (the largest
//                    normalised weight when the side's weights are folded
//                    into the exponent, else 1); packed weights are a / m
//   [6+4DP + side]   D <= 3 layout: 1 when the side's weights are folded
//                    (all >= 0, some > 0, no sigma gradient), 2 when they are
//                    moreover all equal (a~ = 1 on every point), else 0
__host__ __device__ __forceinline__ int meta_stride(int DP) { return 8 + 4 * DP; }
__host__ __device__ __forceinline__ int meta_wscale(int DP) { return 4 + 4 * DP; }
__host__ __device__ __forceinline__ int meta_fold(int DP) { return 6 + 4 * DP; }

// Partial-sum record of one chunk (fp64): [0] sum of effective weights,
// [1] valid points, [2] last valid index (-1: none), [3, 3+DP) sum w' p,
// [3+DP, 3+2DP) sum p over the valid points, [3+2DP] largest and [4+2DP]
// smallest effective weight (D <= 3 layout only).  The backward epilogue
// reuses the same slots for its (Q, R[DP]) partials.
__host__ __device__ __forceinline__ int stats_stride(int DP) { return 5 + 2 * DP; }

// Reduction width: power of two >= D (at least 4); thread (pl, d) of a CTA
// handles dimension d of point lane pl.
__host__ __device__ __forceinline__ int red_width(int D) {
  int r = 4;
  while (r < D) r <<= 1;
  return r;
}

struct PrepArgs {
  int64_t P;
  int D, DP;     // DP: 3 for the D <= 3 path, else the padded generic width
  int layout;    // 0 ragged, 1 dense
  int wmode_x, wmode_y, center;
  int64_t num_x, num_y, nmax_x, nmax_y;
  int64_t chunk_cap;  // capacity of the chunk records (host bound)
  float scale;   // sqrt(log2(e) / (2 sigma^2)): packed coords are scale * (p - anchor)
  const double *sigma_p;  // [P] per-pair bandwidths, or null: `scale` for every pair
  const float *x, *y, *w_x, *w_y;
  const int64_t *ptr_x, *ptr_y;
  const uint8_t *mask_x, *mask_y;
  Seg *seg;
  double *meta;
  double *rec;    // [chunk_cap][stats_stride]
  int64_t *chcnt, *chx, *choff;  // [P], [P], [P + 1]
  int *err;
  int allow_fold;  // D <= 3: weights may be folded into the exponent (no sigma gradient)
  // generic layout (D >= 4): coords [num * DP] (zero padded) and weights [num]
  float *Gx, *Gy, *Ax, *Ay;
};

// The coordinate pre-scale of pair p.
__device__ __forceinline__ float pair_scale(float scale, const double *sigma_p, int64_t p) {
  return sigma_p != nullptr ? scale_of_sigma(sigma_p[p]) : scale;
}

// Effective (masked, raw) weight of point i.
__device__ __forceinline__ float eff_weight(const float *w, const uint8_t *mask, int wmode,
                                            int64_t i) {
  float v = (wmode == 3 || w == nullptr) ? 1.0f : w[i];
  if (mask != nullptr && mask[i] == 0) v = 0.0f;
  return v;
}

// Segment bounds, chunk counts and the chunk map; one CTA of 1024 threads.
// Ragged bounds come from the running maximum of ptr, clamped to [0, num]:
// for a valid ptr that is ptr itself, and for a malformed one (reported
// through the error word) the segments still never overlap, so every bound
// the host derived from num_x and num_y holds.
__global__ void __launch_bounds__(1024) segment_kernel(PrepArgs A) {
  __shared__ int64_t warp_tot[32];
  __shared__ int64_t carry;
  const int tid = threadIdx.x;
  int e = 0;
  for (int side = 0; side < 2; ++side) {
    const int64_t *ptr = side == 0 ? A.ptr_x : A.ptr_y;
    const int64_t num = side == 0 ? A.num_x : A.num_y;
    const int64_t nmax = side == 0 ? A.nmax_x : A.nmax_y;
    if (tid == 0) carry = INT64_MIN;
    __syncthreads();
    for (int64_t base = 0; base < A.P; base += 1024) {
      const int64_t p = base + tid;
      int64_t s, span;
      if (A.layout == 0) {
        const int64_t v = p < A.P ? ptr[p] : INT64_MIN;
        const int64_t pm = block_scan_step<true>(v, warp_tot, &carry);  // max(ptr[0..p])
        if (p >= A.P) continue;
        const int64_t nxt = ptr[p + 1];
        if (p == 0 && v != 0) e |= kErrPtrStart;
        if (p == A.P - 1 && nxt != num) e |= kErrPtrEnd;
        if (nxt < v) e |= kErrPtrOrder;
        int64_t a0 = pm, a1 = nxt > pm ? nxt : pm;
        a0 = a0 < 0 ? 0 : (a0 > num ? num : a0);
        a1 = a1 < 0 ? 0 : (a1 > num ? num : a1);
        s = a0;
        span = a1 - a0;
      } else {
        if (p >= A.P) continue;
        s = p * nmax;
        span = nmax;
      }
      Seg &sg = A.seg[p];
      if (side == 0) {
        sg.xs = s;
        sg.xspan = span;
        A.chx[p] = ceil_div(span, (int64_t)kChunk);
      } else {
        sg.ys = s;
        sg.yspan = span;
        A.chcnt[p] = A.chx[p] + ceil_div(span, (int64_t)kChunk);
      }
    }
    __syncthreads();
  }
  if (e) atomicOr(A.err, e);
  block_exclusive_scan(A.chcnt, A.choff, A.P, A.chunk_cap, warp_tot, &carry);
}

// Pass 1: per-chunk partial sums of weights and coordinates.
template <int NT>
__global__ void __launch_bounds__(NT) stats_kernel(PrepArgs A) {
  __shared__ double sh[NT];
  __shared__ int64_t shl[NT];
  const ChunkMap M{A.P, A.choff, A.chx};
  const int tid = threadIdx.x;
  const int D = A.D, DP = A.DP;
  const int RW = red_width(D);
  const int lanes = NT / RW;
  const int d = tid % RW, pl = tid / RW;
  for_each_chunk(M, [&](int64_t p, int side, int64_t c, int64_t v, int64_t, int64_t) {
    const float *pts = side == 0 ? A.x : A.y;
    const float *w = side == 0 ? A.w_x : A.w_y;
    const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
    const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
    const Seg sg = A.seg[p];
    const int64_t s = side == 0 ? sg.xs : sg.ys;
    const int64_t span = side == 0 ? sg.xspan : sg.yspan;
    const int64_t b = c * kChunk, e = b + kChunk < span ? b + kChunk : span;
    double acc = 0.0, accu = 0.0, wsum = 0.0;
    int64_t last = -1, nvalid = 0;
    for (int64_t i = b + pl; i < e; i += lanes) {
      const int64_t g = s + i;
      const float wi = eff_weight(w, mask, wmode, g);
      const bool valid = mask == nullptr || mask[g] != 0;
      if (d < D) {
        const double val = (double)pts[g * D + d];
        acc += (double)wi * val;
        if (valid) accu += val;
      }
      if (d == 0) {
        wsum += (double)wi;
        if (valid) {
          last = i;
          ++nvalid;
        }
      }
    }
    double *rec = A.rec + v * stats_stride(DP);
    // coordinate sums: reduce over the point lanes in lane order
    sh[tid] = acc;
    __syncthreads();
    if (tid < DP) {
      double t = 0.0;
      for (int l = 0; l < lanes; ++l) t += sh[l * RW + tid];
      rec[3 + tid] = t;
    }
    __syncthreads();
    sh[tid] = accu;
    __syncthreads();
    if (tid < DP) {
      double t = 0.0;
      for (int l = 0; l < lanes; ++l) t += sh[l * RW + tid];
      rec[3 + DP + tid] = t;
    }
    __syncthreads();
    sh[tid] = wsum;
    shl[tid] = last;
    __syncthreads();
    if (tid == 0) {
      double W = 0.0;
      int64_t lst = -1;
      for (int l = 0; l < lanes; ++l) {
        W += sh[l * RW];
        lst = shl[l * RW] > lst ? shl[l * RW] : lst;
      }
      rec[0] = W;
      rec[2] = (double)lst;
    }
    __syncthreads();
    shl[tid] = nvalid;
    __syncthreads();
    if (tid == 0) {
      int64_t nv = 0;
      for (int l = 0; l < lanes; ++l) nv += shl[l * RW];
      rec[1] = (double)nv;
    }
    __syncthreads();
  });
}

// Pass 1 for D <= 3: one thread per point, all nine partial sums reduced at
// once (shuffle trees, then the 8 warps in order) -- one barrier pair per
// chunk instead of the generic kernel's three lane-serial reductions.
template <int NT>
__global__ void __launch_bounds__(NT) stats3_kernel(PrepArgs A) {
  __shared__ double sh[(NT / 32) * 8];
  __shared__ long long shl[NT / 32];
  __shared__ double shm[NT / 32][2];
  const ChunkMap M{A.P, A.choff, A.chx};
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int D = A.D;
  for_each_chunk(M, [&](int64_t p, int side, int64_t c, int64_t v, int64_t, int64_t) {
    const float *pts = side == 0 ? A.x : A.y;
    const float *w = side == 0 ? A.w_x : A.w_y;
    const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
    const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
    const Seg sg = A.seg[p];
    const int64_t s = side == 0 ? sg.xs : sg.ys;
    const int64_t span = side == 0 ? sg.xspan : sg.yspan;
    const int64_t b = c * kChunk, e = b + kChunk < span ? b + kChunk : span;
    // vals: W, valid count, sum w' p (3), sum p over valid points (3)
    double vals[8] = {0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0};
    long long last = -1;
    double wmax = -INFINITY, nwmin = -INFINITY;
    for (int64_t i = b + tid; i < e; i += NT) {
      const int64_t g = s + i;
      const float wi = eff_weight(w, mask, wmode, g);
      const bool valid = mask == nullptr || mask[g] != 0;
      vals[0] += (double)wi;
      wmax = fmax(wmax, (double)wi);
      nwmin = fmax(nwmin, -(double)wi);
#pragma unroll
      for (int d = 0; d < 3; ++d) {
        if (d < D) {
          const double pv = (double)pts[g * D + d];
          vals[2 + d] += (double)wi * pv;
          if (valid) vals[5 + d] += pv;
        }
      }
      if (valid) {
        vals[1] += 1.0;
        last = i;
      }
    }
    last = warp_max(last);
    wmax = warp_fmax(wmax);
    nwmin = warp_fmax(nwmin);
    if (lane == 0) {
      shl[wid] = last;
      shm[wid][0] = wmax;
      shm[wid][1] = nwmin;
    }
    block_sum_n<8>(vals, sh);  // its first barrier also publishes shl and shm
    if (tid == 0) {
      double *rec = A.rec + v * stats_stride(3);
      long long lst = -1;
      double mx = -INFINITY, nmn = -INFINITY;
      for (int k = 0; k < NT / 32; ++k) {
        lst = shl[k] > lst ? shl[k] : lst;
        mx = fmax(mx, shm[k][0]);
        nmn = fmax(nmn, shm[k][1]);
      }
      rec[9] = mx;
      rec[10] = -nmn;
      rec[0] = vals[0];
      rec[1] = vals[1];
      rec[2] = (double)lst;
#pragma unroll
      for (int d = 0; d < 3; ++d) {
        rec[3 + d] = vals[2 + d];
        rec[6 + d] = vals[5 + d];
      }
    }
    // the next chunk's shl / shm writes happen after block_sum_n's trailing barrier
  });
}

// Pass 1 for wide points (DP >= 32): one warp per point, lane l holding
// coordinates l, l + 32, ...; a chunk's partials are combined over the 8
// warps in order through shared memory, one barrier pair per chunk.
template <int DP>
__global__ void __launch_bounds__(256) statsw_kernel(PrepArgs A) {
  constexpr int NW = 8, KL = DP / 32;
  __shared__ double sh[NW][2 * DP + 2];
  __shared__ long long shl[NW];
  const ChunkMap M{A.P, A.choff, A.chx};
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int D = A.D;
  for_each_chunk(M, [&](int64_t p, int side, int64_t c, int64_t v, int64_t, int64_t) {
    const float *pts = side == 0 ? A.x : A.y;
    const float *w = side == 0 ? A.w_x : A.w_y;
    const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
    const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
    const Seg sg = A.seg[p];
    const int64_t s = side == 0 ? sg.xs : sg.ys;
    const int64_t span = side == 0 ? sg.xspan : sg.yspan;
    const int64_t b = c * kChunk, e = b + kChunk < span ? b + kChunk : span;
    double acc[KL], accu[KL], W = 0.0, nv = 0.0;
    long long last = -1;
#pragma unroll
    for (int k = 0; k < KL; ++k) acc[k] = accu[k] = 0.0;
    for (int64_t i = b + wid; i < e; i += NW) {
      const int64_t g = s + i;
      const float wi = eff_weight(w, mask, wmode, g);
      const bool valid = mask == nullptr || mask[g] != 0;
#pragma unroll
      for (int k = 0; k < KL; ++k) {
        const int d = lane + 32 * k;
        if (d < D) {
          const double pv = (double)pts[g * D + d];
          acc[k] += (double)wi * pv;
          if (valid) accu[k] += pv;
        }
      }
      W += (double)wi;
      if (valid) {
        nv += 1.0;
        last = i;
      }
    }
#pragma unroll
    for (int k = 0; k < KL; ++k) {
      sh[wid][lane + 32 * k] = acc[k];
      sh[wid][DP + lane + 32 * k] = accu[k];
    }
    if (lane == 0) {
      sh[wid][2 * DP] = W;
      sh[wid][2 * DP + 1] = nv;
      shl[wid] = last;
    }
    __syncthreads();
    double *rec = A.rec + v * stats_stride(DP);
    for (int t = tid; t < 2 * DP + 2; t += 256) {
      double tot = 0.0;
      for (int q = 0; q < NW; ++q) tot += sh[q][t];
      if (t < 2 * DP) rec[3 + t] = tot;  // sum w' p, then sum p (valid points)
      else rec[t - 2 * DP] = tot;        // W, valid count
    }
    if (tid == 0) {
      long long lst = -1;
      for (int q = 0; q < NW; ++q) lst = shl[q] > lst ? shl[q] : lst;
      rec[2] = (double)lst;
    }
    __syncthreads();
  });
}

__device__ __forceinline__ double warp_max(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

// Pass 2: one warp per pair combines its chunk records into the segment
// bounds and normalisers (lane-strided over the chunks, then a fixed shuffle
// tree) and the centroids and anchors (one lane per coordinate, the chunks in
// order).
__global__ void __launch_bounds__(128) meta_kernel(PrepArgs A) {
  const int64_t p = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (p >= A.P) return;
  const int D = A.D, DP = A.DP;
  if (A.sigma_p != nullptr && lane == 0 && !(A.sigma_p[p] > 0.0)) atomicOr(A.err, (int)kErrSigma);
  const int rs = stats_stride(DP);
  double *meta = A.meta + p * meta_stride(DP);
  const int64_t lo = A.choff[p], hi = A.choff[p + 1];
  int64_t cxn = A.chx[p];
  if (cxn > hi - lo) cxn = hi - lo;
  int64_t count_x = 0;
  for (int side = 0; side < 2; ++side) {
    const int64_t first = side == 0 ? lo : lo + cxn;
    const int64_t n = side == 0 ? cxn : (hi - lo) - cxn;
    const double *r0 = A.rec + first * rs;
    double W = 0.0, nv = 0.0, lst = -1.0;
    for (int64_t c = lane; c < n; c += 32) {
      W += r0[c * rs + 0];
      nv += r0[c * rs + 1];
      lst = fmax(lst, r0[c * rs + 2]);
    }
    W = warp_sum(W);
    nv = warp_sum(nv);
    lst = warp_max(lst);
    const int64_t span = side == 0 ? A.seg[p].xspan : A.seg[p].yspan;
    const int64_t count = A.layout == 0 ? span : (int64_t)lst + 1;
    const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
    double Wn;
    if (wmode == 0) {
      Wn = 1.0;  // raw weights
    } else if (wmode == 3) {
      Wn = nv > 0 ? nv : 1.0;  // uniform 1/count
    } else if (wmode == 2) {
      Wn = W > 1e-8 ? W : 1e-8;  // clamp_min(1e-8)
    } else {
      Wn = W;
      if (lane == 0 && count > 0 && !(W > 0.0) && !(W != W)) atomicOr(A.err, (int)kErrWeightSum);
      if (!(W > 0.0)) Wn = 1.0;  // keep the kernels finite; the error is reported
    }
    // D <= 3: fold the weights into the exponent when they are all >= 0
    // (k' = 2^(-(r^2 - log2(a / m))) = (a / m) k, m the largest weight)
    double m = 1.0, fold = 0.0;
    if (DP == 3) {
      double wmax = -INFINITY, nwmin = -INFINITY;
      for (int64_t c = lane; c < n; c += 32) {
        wmax = fmax(wmax, r0[c * rs + 9]);
        nwmin = fmax(nwmin, -r0[c * rs + 10]);
      }
      wmax = warp_fmax(wmax);
      nwmin = warp_fmax(nwmin);
      if (A.allow_fold && -nwmin >= 0.0 && wmax > 0.0 && Wn > 0.0 && wmax / Wn < INFINITY) {
        m = wmax / Wn;
        fold = -nwmin == wmax ? 2.0 : 1.0;
      }
    }
    if (lane == 0) {
      meta[side] = Wn;
      meta[2 + side] = W;
      meta[meta_wscale(DP) + side] = m;
      meta[meta_fold(DP) + side] = fold;
      if (side == 0) A.seg[p].xcount = count;
      else A.seg[p].ycount = count;
    }
    if (side == 0) count_x = count;
    // one lane per coordinate, the chunks summed in order (fixed order:
    // deterministic); each lane also finishes its own coordinates below
    for (int dd = lane; dd < DP; dd += 32) {
      double cs = 0.0, ps = 0.0;
      for (int64_t c = 0; c < n; ++c) {
        cs += r0[c * rs + 3 + dd];
        ps += r0[c * rs + 3 + DP + dd];
      }
      {
        // centroid mu = sum_i a_i p_i = sum_i w'_i p_i / Wn; plain mean for the anchor
        const double mu = dd < D ? cs / Wn : 0.0;
        const double mean = (dd < D && nv > 0) ? ps / nv : 0.0;
        meta[4 + side * DP + dd] = mu;
        if (side == 0) {
          meta[4 + 2 * DP + dd] = mean;  // provisional: replaced by the anchor below
        } else {
          // anchors.  Centering: each cloud is shifted by its weighted
          // centroid (the semantics).  Otherwise both clouds share one anchor,
          // the unweighted mean of the valid x points (of the y points when x
          // has none): distances do not change, and the packed coordinates
          // stay as small as the clouds themselves whatever the weights are.
          double ax, ay;
          if (A.center) {
            ax = meta[4 + dd];
            ay = mu;
          } else {
            ax = count_x > 0 ? meta[4 + 2 * DP + dd] : mean;
            ay = ax;
          }
          meta[4 + 2 * DP + dd] = ax;
          meta[4 + 3 * DP + dd] = ay;
        }
      }
    }
  }
}

// Generic layout (D >= 4): scaled, anchored coordinates and normalised weights.
template <int NT>
__global__ void __launch_bounds__(NT) packg_kernel(PrepArgs A) {
  const ChunkMap M{A.P, A.choff, A.chx};
  const int D = A.D, DP = A.DP;
  const int RW = red_width(D);
  const int lanes = NT / RW;
  const int d = threadIdx.x % RW, pl = threadIdx.x / RW;
  for_each_chunk(M, [&](int64_t p, int side, int64_t c, int64_t, int64_t, int64_t) {
    const Seg sg = A.seg[p];
    const int64_t s = side == 0 ? sg.xs : sg.ys;
    const int64_t count = side == 0 ? sg.xcount : sg.ycount;
    const float *pts = side == 0 ? A.x : A.y;
    const float *w = side == 0 ? A.w_x : A.w_y;
    const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
    const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
    float *Gp = side == 0 ? A.Gx : A.Gy;
    float *Ap = side == 0 ? A.Ax : A.Ay;
    const double *meta = A.meta + p * meta_stride(DP);
    const double Wn = meta[side];
    const double *anc = meta + 4 + (2 + side) * DP;
    const float sc = pair_scale(A.scale, A.sigma_p, p);
    const int64_t b = c * kChunk, e = b + kChunk < count ? b + kChunk : count;
    for (int64_t i = b + pl; i < e; i += lanes) {
      const int64_t g = s + i;
      if (d < DP) {
        float val = 0.f;
        if (d < D) val = sc * (float)((double)pts[g * D + d] - anc[d]);
        Gp[g * DP + d] = val;
      }
      if (d == 0) Ap[g] = (float)((double)eff_weight(w, mask, wmode, g) / Wn);
    }
  });
}

// Generic layout for wide points (DP >= 32, D a multiple of 4): float4
// elements (point, coordinates 4c..4c+3) taken flat.  With 256 threads and
// DP / 4 dividing 256, a thread always handles the same c, so its four
// anchors are loaded once per pair side.
template <int DP>
__global__ void __launch_bounds__(256, 4) packgw_kernel(PrepArgs A) {
  constexpr int NC = DP / 4;  // float4 chunks per packed point
  static_assert(256 % NC == 0, "a thread keeps one chunk");
  const ChunkMap M{A.P, A.choff, A.chx};
  const int D = A.D, c = threadIdx.x % NC;
  for_each_chunk(M, [&](int64_t p, int side, int64_t ch, int64_t, int64_t, int64_t) {
    const Seg sg = A.seg[p];
    const int64_t s = side == 0 ? sg.xs : sg.ys;
    const int64_t count = side == 0 ? sg.xcount : sg.ycount;
    const float *pts = side == 0 ? A.x : A.y;
    const float *w = side == 0 ? A.w_x : A.w_y;
    const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
    const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
    float4 *Gp = reinterpret_cast<float4 *>(side == 0 ? A.Gx : A.Gy);
    float *Ap = side == 0 ? A.Ax : A.Ay;
    const double *meta = A.meta + p * meta_stride(DP);
    const double Wn = meta[side];
    const double *anc = meta + 4 + (2 + side) * DP;
    const bool live = 4 * c < D;
    // anchors kept in fp64: the same packed values as the scalar kernel
    const double a0 = live ? anc[4 * c] : 0.0, a1 = live ? anc[4 * c + 1] : 0.0;
    const double a2 = live ? anc[4 * c + 2] : 0.0, a3 = live ? anc[4 * c + 3] : 0.0;
    const float sc = pair_scale(A.scale, A.sigma_p, p);
    const int64_t b = ch * kChunk, e = b + kChunk < count ? b + kChunk : count;
    const int64_t nel = (e - b) * NC;
    for (int64_t k0 = threadIdx.x; k0 < nel; k0 += 4 * 256) {
      // the 4 loads go out before the first store (a store to Gp might
      // alias pts as far as the compiler knows, which would serialise them)
      float4 xv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t k = k0 + u * 256;
        xv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (k < nel && live)
          xv[u] = *reinterpret_cast<const float4 *>(pts + (s + b + k / NC) * D + 4 * c);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t k = k0 + u * 256;
        if (k < nel) {
          const float4 x = xv[u];
          Gp[(s + b + k / NC) * NC + c] =
              live ? make_float4(sc * (float)((double)x.x - a0), sc * (float)((double)x.y - a1),
                                 sc * (float)((double)x.z - a2), sc * (float)((double)x.w - a3))
                   : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
    // normalised weights, one point per thread
    for (int64_t i = b + threadIdx.x; i < e; i += 256)
      Ap[s + i] = (float)((double)eff_weight(w, mask, wmode, s + i) / Wn);
  });
}

// ---------------------------------------------------------------------------
// D <= 3 tile layout.  Each cloud is cut into 64-point tiles, zero-weight
// padded; pair p's x tiles start at tile tbase_x[p] (exclusive scan of
// ceil(count / 64)).  A tile stores two arrays of 64 duplicated pairs
// (16 bytes per point each):  {x', x', y', y'}  and  {z', z', v, v}
// so one column feeds packed f32x2 arithmetic against two rows, and a warp
// reads any column of a tile at an immediate offset from the tile base.
// With m the side's weight scale and a~ = a / m (also stored alone, per
// slot, in aw_x / aw_y), v is -log2(a~) for a side whose weights are folded
// into the exponent (64 for a zero weight, +inf for padding) and a~ itself
// otherwise.  On a side with equal weights (a~ = 1) the padding slots sit at
// coordinate 1e18, so that as rows they give k = 0 without the weight
// (valid while the scaled coordinates |x'| stay far below that).
// ---------------------------------------------------------------------------
struct PackArgs {
  int64_t P;
  int D, nq;
  float scale;
  const double *sigma_p;  // [P] per-pair bandwidths, or null
  const float *x, *y, *w_x, *w_y;
  const uint8_t *mask_x, *mask_y;
  int wmode_x, wmode_y;
  const Seg *seg;
  const double *meta;
  const int64_t *choff, *chx;
  const int64_t *tbase_x, *tbase_y;  // [P + 1]
  int64_t max_tiles_x, max_tiles_y;
  ulonglong2 *tiles_x, *tiles_y;     // [tiles][nq = 2][64]
  float *aw_x, *aw_y;                // [tiles * 64] a~ per slot
};

template <int NT>
__global__ void __launch_bounds__(NT) pack3_kernel(PackArgs A) {
  const ChunkMap M{A.P, A.choff, A.chx};
  for_each_chunk(M, [&](int64_t p, int side, int64_t c, int64_t, int64_t, int64_t) {
    const Seg sg = A.seg[p];
    const int D = A.D;
    const int64_t s = side == 0 ? sg.xs : sg.ys;
    const int64_t count = side == 0 ? sg.xcount : sg.ycount;
    const int64_t t0 = (side == 0 ? A.tbase_x : A.tbase_y)[p];
    const int64_t t1 = (side == 0 ? A.tbase_x : A.tbase_y)[p + 1];
    const int64_t tmax = side == 0 ? A.max_tiles_x : A.max_tiles_y;
    const float *pts = side == 0 ? A.x : A.y;
    const float *w = side == 0 ? A.w_x : A.w_y;
    const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
    const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
    ulonglong2 *tiles = side == 0 ? A.tiles_x : A.tiles_y;
    float *aw = side == 0 ? A.aw_x : A.aw_y;
    const double *meta = A.meta + p * meta_stride(3);
    const double Wm = meta[side] * meta[meta_wscale(3) + side];  // a~ = w' / Wm
    const bool fold = meta[meta_fold(3) + side] != 0.0;
    const bool uni = meta[meta_fold(3) + side] == 2.0;
    const float pad = uni ? 1e18f : 0.f;
    const float ax = (float)meta[4 + (2 + side) * 3 + 0];
    const float ay = (float)meta[4 + (2 + side) * 3 + 1];
    const float az = (float)meta[4 + (2 + side) * 3 + 2];
    const float scale = pair_scale(A.scale, A.sigma_p, p);
    const int nq = A.nq;
    const int64_t npad = (t1 - t0) * kTile;
    const int64_t b = c * kChunk, e = b + kChunk < npad ? b + kChunk : npad;
    for (int64_t i = b + threadIdx.x; i < e; i += NT) {
      const int64_t t = t0 + i / kTile;
      if (t >= tmax) break;  // malformed ptr overflowing the bound (error already flagged)
      float c0 = pad, c1 = pad, c2 = pad, a = 0.f, v = fold ? INFINITY : 0.f;
      if (i < count) {
        const int64_t g = s + i;
        const double at = uni ? 1.0 : (double)eff_weight(w, mask, wmode, g) / Wm;
        a = (float)at;
        c1 = c2 = 0.f;
        // folded: a~ in [0, 1]; a zero weight becomes 2^-64, which leaves the
        // other points' sums unchanged to 5e-20 and keeps the point's own
        // row sums (its weight gradient) finite
        v = fold ? (at >= 1.0 ? 0.f : at > 0x1p-64 ? (float)-log2(at) : 64.f) : a;
        c0 = scale * (pts[g * D + 0] - ax);
        if (D > 1) c1 = scale * (pts[g * D + 1] - ay);
        if (D > 2) c2 = scale * (pts[g * D + 2] - az);
      }
      ulonglong2 *tp = tiles + t * (int64_t)(nq * kTile) + (i % kTile);
      tp[0] = make_ulonglong2(pk2u(c0, c0), pk2u(c1, c1));
      tp[kTile] = make_ulonglong2(pk2u(c2, c2), pk2u(v, v));
      aw[t * (int64_t)kTile + (i % kTile)] = a;
    }
  });
}

}  // namespace ra
