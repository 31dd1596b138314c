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

#include <cuda_fp16.h>

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
//   [8+4DP + side]   tensor-core layout (fp16 tiles): 2^e, the power of two
//                    the side's packed coordinates are multiplied by before
//                    the fp16 split (their magnitude bound times 2^e <= 2^15)
//   [10+4DP + side]  tensor-core layout: 2^-f, the power of two the side's
//                    normalised weights are multiplied by (largest |a| 2^-f
//                    in (1/2, 1])
//   [12+4DP + side]  tensor-core layout: 1 when the side's weights are all
//                    >= 0 (folded into the exponent as columns), else 0
//   [14+4DP, 14+6DP) tensor-core layout: the anchors as fp32 pairs (hi, lo
//                    with hi + lo = anchor to ~48 bits), floats [side][2][DP]:
//                    x' = c ((x - hi) - lo) in fp32 without fp64 conversions
__host__ __device__ __forceinline__ int meta_stride(int DP) { return 14 + 6 * DP; }
__host__ __device__ __forceinline__ int meta_wscale(int DP) { return 4 + 4 * DP; }
__host__ __device__ __forceinline__ int meta_fold(int DP) { return 6 + 4 * DP; }
__host__ __device__ __forceinline__ int meta_tc_cscale(int DP) { return 8 + 4 * DP; }
__host__ __device__ __forceinline__ int meta_tc_wscale(int DP) { return 10 + 4 * DP; }
__host__ __device__ __forceinline__ int meta_tc_fold(int DP) { return 12 + 4 * DP; }
__host__ __device__ __forceinline__ int meta_tc_anchor(int DP) { return 14 + 4 * DP; }
// x' = c ((x - hi) - lo) from a side's fp32 anchor pairs (tensor-core layout)
__device__ __forceinline__ const float *tc_anchor(const double *meta, int DP, int side) {
  return reinterpret_cast<const float *>(meta + meta_tc_anchor(DP)) + side * 2 * DP;
}

// Partial-sum record of one chunk (fp64): [0] sum of effective weights,
// [1] valid points, [2] last valid index (-1: none), [3, 3+DP) sum w' p,
// [3+DP, 3+2DP) sum p over the valid points, [3+2DP] largest and [4+2DP]
// smallest effective weight (D <= 3 layout, and the wide generic passes),
// [5+2DP] largest |coordinate| of a valid point (wide generic passes).  The
// backward epilogue reuses the same slots for its (Q, R[DP]) partials.
__host__ __device__ __forceinline__ int stats_stride(int DP) { return 6 + 2 * DP; }

// Reduction width: power of two >= D (at least 4); thread (pl, d) of a CTA
// handles dimension d of point lane pl.
__host__ __device__ __forceinline__ int red_width(int D) {
  int r = 4;
  while (r < D) r <<= 1;
  return r;
}

// D <= 3: a pair with at most kSmallPts points on each side (span) is
// prepared by one CTA of prep3_kernel (sums, metadata and packing in one
// pass over its points); larger pairs take the chunked passes stats3_kernel,
// meta_kernel and pack3_kernel, which spread one pair over many CTAs.
constexpr int64_t kSmallPts = 4096;
__host__ __device__ __forceinline__ bool small_pair(const Seg &s) {
  return s.xspan <= kSmallPts && s.yspan <= kSmallPts;
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
  int32_t *cpair;                // [chunk_cap]: pair of each virtual chunk
  unsigned *ticket;              // chunk counter of the launch (ra_chunks.cuh), zeroed
  unsigned *pair_ticket;         // pair counter of prep3_kernel, zeroed
  int64_t *tcnt;                 // [2P] scratch: 64-point tiles of each side (D <= 3)
  int64_t *tbase_x, *tbase_y;    // [P + 1]: first tile of each pair's cloud (D <= 3)
  int *err;
  int allow_fold;  // D <= 3: weights may be folded into the exponent (no sigma gradient)
  // generic layout (D >= 4): coords [num * DP] (zero padded) and weights [num]
  float *Gx, *Gy, *Ax, *Ay;
  // tensor-core layout (ra_tc16.cuh): fp16 hi / lo tiles of 64 points and
  // kT16SlotFloats slot values per tile, from tile tbase_x / tbase_y of a pair
  int tc16;
  uint8_t *hx, *hy, *lx, *ly;
  float *cx, *cy;
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

// cpair[v] = the pair of virtual chunk v, once choff is complete (the
// segment kernel's CTA, after a barrier).
__device__ __forceinline__ void chunk_pairs(const PrepArgs &A) {
  const ChunkMap M{A.P, A.choff, A.chx};
  const int64_t total = A.choff[A.P];
  for (int64_t v = threadIdx.x; v < total; v += blockDim.x) A.cpair[v] = (int32_t)chunk_pair(M, v);
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
        // D <= 3: the chunk map covers only the pairs the chunked passes
        // prepare (small pairs have their own one-CTA kernels)
        if (A.DP == 3 && A.tcnt != nullptr && small_pair(sg)) A.chx[p] = A.chcnt[p] = 0;
      }
      // tile layouts (D <= 3, tensor-core): room for the whole span (a dense
      // row's count, 1 + its last valid index, is known only after the sums)
      if (A.tcnt != nullptr) A.tcnt[side * A.P + p] = ceil_div(span, (int64_t)kTile);
    }
    __syncthreads();
  }
  if (e) atomicOr(A.err, e);
  if (A.tcnt == nullptr) {
    block_exclusive_scan(A.chcnt, A.choff, A.P, A.chunk_cap, warp_tot, &carry);
    chunk_pairs(A);
    return;
  }
  // the chunk map and both tile bases in one pass over the pairs
  __shared__ int64_t warp_tot3[3][32];
  __shared__ int64_t carry3[3];
  if (tid < 3) carry3[tid] = 0;
  __syncthreads();
  const int lane = tid & 31, wid = tid >> 5;
  for (int64_t base = 0; base < A.P; base += 1024) {
    const int64_t p = base + tid;
    const bool in = p < A.P;
    const int64_t v[3] = {in ? A.chcnt[p] : 0, in ? A.tcnt[p] : 0, in ? A.tcnt[A.P + p] : 0};
    int64_t inc[3] = {v[0], v[1], v[2]};
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        const int64_t t = __shfl_up_sync(kFull, inc[k], o);
        if (lane >= o) inc[k] += t;
      }
    }
    if (lane == 31) {
#pragma unroll
      for (int k = 0; k < 3; ++k) warp_tot3[k][wid] = inc[k];
    }
    __syncthreads();
    if (wid == 0) {
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        int64_t t = warp_tot3[k][lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int64_t u = __shfl_up_sync(kFull, t, o);
          if (lane >= o) t += u;
        }
        warp_tot3[k][lane] = t;  // inclusive over warps
      }
    }
    __syncthreads();
    int64_t r[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) r[k] = inc[k] + (wid > 0 ? warp_tot3[k][wid - 1] : 0) + carry3[k];
    if (in) {
      const int64_t e0 = r[0] - v[0];
      A.choff[p] = e0 < A.chunk_cap ? e0 : A.chunk_cap;
      A.tbase_x[p] = r[1] - v[1];
      A.tbase_y[p] = r[2] - v[2];
    }
    __syncthreads();
    if (tid == 1023) {
#pragma unroll
      for (int k = 0; k < 3; ++k) carry3[k] = r[k];
    }
    __syncthreads();
  }
  if (tid == 0) {
    A.choff[A.P] = carry3[0] < A.chunk_cap ? carry3[0] : A.chunk_cap;
    A.tbase_x[A.P] = carry3[1];
    A.tbase_y[A.P] = carry3[2];
  }
  __syncthreads();
  chunk_pairs(A);
}

// Pass 1: per-chunk partial sums of weights and coordinates.
template <int NT>
__global__ void __launch_bounds__(NT) stats_kernel(PrepArgs A) {
  __shared__ double sh[NT];
  __shared__ int64_t shl[NT];
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
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
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int D = A.D;
  for_each_chunk(M, [&](int64_t p, int side, int64_t c, int64_t v, int64_t, int64_t) {
    const float *pts = side == 0 ? A.x : A.y;
    const float *w = side == 0 ? A.w_x : A.w_y;
    const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
    const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
    const Seg sg = A.seg[p];
    if (small_pair(sg)) return;  // prepared by prep3_kernel
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
  __shared__ float shm[NW][3];
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
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
    float wmax = -INFINITY, wmin = INFINITY, cmax = 0.f;
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
          const float pf = pts[g * D + d];
          const double pv = (double)pf;
          acc[k] += (double)wi * pv;
          if (valid) {
            accu[k] += pv;
            cmax = fmaxf(cmax, fabsf(pf));
          }
        }
      }
      W += (double)wi;
      wmax = fmaxf(wmax, wi);
      wmin = fminf(wmin, wi);
      if (valid) {
        nv += 1.0;
        last = i;
      }
    }
    wmax = warp_fmaxf(wmax);
    wmin = -warp_fmaxf(-wmin);
    cmax = warp_fmaxf(cmax);
#pragma unroll
    for (int k = 0; k < KL; ++k) {
      sh[wid][lane + 32 * k] = acc[k];
      sh[wid][DP + lane + 32 * k] = accu[k];
    }
    if (lane == 0) {
      sh[wid][2 * DP] = W;
      sh[wid][2 * DP + 1] = nv;
      shl[wid] = last;
      shm[wid][0] = wmax;
      shm[wid][1] = wmin;
      shm[wid][2] = cmax;
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
      float m0 = -INFINITY, m1 = INFINITY, m2 = 0.f;
      for (int q = 0; q < NW; ++q) {
        lst = shl[q] > lst ? shl[q] : lst;
        m0 = fmaxf(m0, shm[q][0]);
        m1 = fminf(m1, shm[q][1]);
        m2 = fmaxf(m2, shm[q][2]);
      }
      rec[2] = (double)lst;
      rec[3 + 2 * DP] = m0;
      rec[4 + 2 * DP] = m1;
      rec[5 + 2 * DP] = m2;
    }
    __syncthreads();
  });
}

// Pass 1 for wide points whose coordinates load as float4 (D % 4 == 0,
// 16-byte aligned bases): LPP lanes share a point (one float4 chunk or two
// each), a warp covers PPW points per step and keeps kU steps of loads in
// flight, so a CTA has 16-32 KB of reads outstanding.  Partials are combined
// over the PPW point slots of a warp by shuffles, then over the 8 warps in
// order: a fixed summation order, independent of scheduling.
template <int DP>
__global__ void __launch_bounds__(256, 2) statsw4_kernel(PrepArgs A) {
  constexpr int NW = 8, NC = DP / 4;
  constexpr int LPP = NC < 32 ? NC : 32;  // lanes per point
  constexpr int CPL = NC / LPP;           // float4 chunks per lane
  constexpr int PPW = 32 / LPP;           // points per warp step
  constexpr int kU = CPL == 1 ? 8 : 4;    // warp steps in flight
  static_assert(NC % LPP == 0 && 32 % LPP == 0, "chunk split");
  __shared__ double sh[NW][2 * DP + 2];
  __shared__ long long shl[NW];
  __shared__ float shm[NW][3];
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int cl = lane % LPP, q = lane / LPP;
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
    double acc[CPL][4], accu[CPL][4], W = 0.0, nv = 0.0;
    long long last = -1;
    float wmax = -INFINITY, wmin = INFINITY, cmax = 0.f;
#pragma unroll
    for (int k = 0; k < CPL; ++k)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[k][j] = accu[k][j] = 0.0;
    constexpr int kStep = NW * PPW;  // points of one CTA step
    for (int64_t i0 = b + wid * PPW + q; i0 < e; i0 += (int64_t)kU * kStep) {
      float4 xv[kU][CPL];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = i0 + (int64_t)u * kStep;
#pragma unroll
        for (int k = 0; k < CPL; ++k) {
          const int cc = cl + LPP * k;
          xv[u][k] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (i < e && 4 * cc < D)
            xv[u][k] = *reinterpret_cast<const float4 *>(pts + (s + i) * D + 4 * cc);
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = i0 + (int64_t)u * kStep;
        if (i < e) {
          const int64_t g = s + i;
          const double wi = (double)eff_weight(w, mask, wmode, g);
          const bool valid = mask == nullptr || mask[g] != 0;
#pragma unroll
          for (int k = 0; k < CPL; ++k) {
            const float xs[4] = {xv[u][k].x, xv[u][k].y, xv[u][k].z, xv[u][k].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const double pv = (double)xs[j];
              acc[k][j] += wi * pv;
              if (valid) {
                accu[k][j] += pv;
                cmax = fmaxf(cmax, fabsf(xs[j]));
              }
            }
          }
          wmax = fmaxf(wmax, (float)wi);
          wmin = fminf(wmin, (float)wi);
          if (cl == 0) {
            W += wi;
            if (valid) {
              nv += 1.0;
              last = i;
            }
          }
        }
      }
    }
    // combine the PPW point slots of the warp (lanes cl, cl + LPP, ...)
#pragma unroll
    for (int o = LPP; o < 32; o <<= 1) {
#pragma unroll
      for (int k = 0; k < CPL; ++k)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[k][j] += __shfl_xor_sync(kFull, acc[k][j], o);
          accu[k][j] += __shfl_xor_sync(kFull, accu[k][j], o);
        }
      W += __shfl_xor_sync(kFull, W, o);
      nv += __shfl_xor_sync(kFull, nv, o);
      const long long lo = __shfl_xor_sync(kFull, last, o);
      last = lo > last ? lo : last;
    }
    if (q == 0) {
#pragma unroll
      for (int k = 0; k < CPL; ++k)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sh[wid][4 * (cl + LPP * k) + j] = acc[k][j];
          sh[wid][DP + 4 * (cl + LPP * k) + j] = accu[k][j];
        }
    }
    wmax = warp_fmaxf(wmax);
    wmin = -warp_fmaxf(-wmin);
    cmax = warp_fmaxf(cmax);
    if (lane == 0) {
      sh[wid][2 * DP] = W;
      sh[wid][2 * DP + 1] = nv;
      shl[wid] = last;
      shm[wid][0] = wmax;
      shm[wid][1] = wmin;
      shm[wid][2] = cmax;
    }
    __syncthreads();
    double *rec = A.rec + v * stats_stride(DP);
    for (int t = tid; t < 2 * DP + 2; t += 256) {
      double tot = 0.0;
      for (int qq = 0; qq < NW; ++qq) tot += sh[qq][t];
      if (t < 2 * DP) rec[3 + t] = tot;  // sum w' p, then sum p (valid points)
      else rec[t - 2 * DP] = tot;        // W, valid count
    }
    if (tid == 0) {
      long long lst = -1;
      float m0 = -INFINITY, m1 = INFINITY, m2 = 0.f;
      for (int qq = 0; qq < NW; ++qq) {
        lst = shl[qq] > lst ? shl[qq] : lst;
        m0 = fmaxf(m0, shm[qq][0]);
        m1 = fminf(m1, shm[qq][1]);
        m2 = fmaxf(m2, shm[qq][2]);
      }
      rec[2] = (double)lst;
      rec[3 + 2 * DP] = m0;  // largest and smallest effective weight
      rec[4 + 2 * DP] = m1;
      rec[5 + 2 * DP] = m2;  // largest |coordinate| of a valid point
    }
    __syncthreads();
  });
}

__device__ __forceinline__ double warp_max(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

// Normaliser of one side's weights (kde.py:20-27, 115-121, 169-199) and,
// for the D <= 3 layout, whether they fold into the exponent: when they are
// all >= 0, k' = 2^(-(r^2 - log2(a / m))) = (a / m) k with m the largest
// normalised weight.  W: sum of the effective weights, nv: valid points,
// count: points the kernels visit, wmax / nwmin: largest weight and largest
// negated weight.  werr: a SUM-normalised side with points sums to <= 0 (the
// normaliser is then 1, which keeps the kernels finite; the error is
// reported).
__device__ __forceinline__ void side_normaliser(int wmode, double W, double nv, int64_t count,
                                                bool may_fold, double wmax, double nwmin,
                                                double &Wn, double &m, double &fold,
                                                bool &werr) {
  werr = false;
  if (wmode == 0) {
    Wn = 1.0;  // raw weights
  } else if (wmode == 3) {
    Wn = nv > 0 ? nv : 1.0;  // uniform 1/count
  } else if (wmode == 2) {
    Wn = W > 1e-8 ? W : 1e-8;  // clamp_min(1e-8)
  } else {
    Wn = W;
    werr = count > 0 && !(W > 0.0) && !(W != W);
    if (!(W > 0.0)) Wn = 1.0;
  }
  m = 1.0;
  fold = 0.0;
  if (may_fold && -nwmin >= 0.0 && wmax > 0.0 && Wn > 0.0 && wmax / Wn < INFINITY) {
    m = wmax / Wn;
    fold = -nwmin == wmax ? 2.0 : 1.0;
  }
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
  if (DP == 3 && small_pair(A.seg[p])) return;  // prepared by prep3_kernel
  if (A.sigma_p != nullptr && lane == 0 && !(A.sigma_p[p] > 0.0)) atomicOr(A.err, (int)kErrSigma);
  const int rs = stats_stride(DP);
  double *meta = A.meta + p * meta_stride(DP);
  const int64_t lo = A.choff[p], hi = A.choff[p + 1];
  int64_t cxn = A.chx[p];
  if (cxn > hi - lo) cxn = hi - lo;
  int64_t count_x = 0;
  double cmax[2] = {0.0, 0.0};  // largest |coordinate| of each side (tensor-core layout)
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
    int64_t count = A.layout == 0 ? span : (int64_t)lst + 1;
    // within [0, span] whatever the records hold (a pass that gave up on a
    // bounded wait leaves them unwritten): later kernels index by it
    if (!(count >= 0)) count = 0;
    if (count > span) count = span;
    const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
    double wmax = -INFINITY, nwmin = -INFINITY;
    if (DP == 3) {
      for (int64_t c = lane; c < n; c += 32) {
        wmax = fmax(wmax, r0[c * rs + 9]);
        nwmin = fmax(nwmin, -r0[c * rs + 10]);
      }
      wmax = warp_fmax(wmax);
      nwmin = warp_fmax(nwmin);
    }
    double Wn, m, fold;
    bool werr;
    side_normaliser(wmode, W, nv, count, DP == 3 && A.allow_fold, wmax, nwmin, Wn, m, fold, werr);
    if (lane == 0 && werr) atomicOr(A.err, (int)kErrWeightSum);
    if (lane == 0) {
      meta[side] = Wn;
      meta[2 + side] = W;
      meta[meta_wscale(DP) + side] = m;
      meta[meta_fold(DP) + side] = fold;
      if (side == 0) A.seg[p].xcount = count;
      else A.seg[p].ycount = count;
    }
    if (side == 0) count_x = count;
    if (A.tc16) {
      // fp16 operand scales (ra_tc16.cuh): weights |a| 2^-f <= 1; the
      // coordinates' bound is finished below, once the anchors are known
      double w0 = -INFINITY, w1 = INFINITY, c0 = 0.0;
      for (int64_t c = lane; c < n; c += 32) {
        w0 = fmax(w0, r0[c * rs + 3 + 2 * DP]);
        w1 = fmin(w1, r0[c * rs + 4 + 2 * DP]);
        c0 = fmax(c0, r0[c * rs + 5 + 2 * DP]);
      }
      w0 = warp_fmax(w0);
      w1 = -warp_fmax(-w1);
      cmax[side] = warp_fmax(c0);
      if (lane == 0) {
        // the largest |a| 2^-f lands in (1/2, 1]: small weights (1/n) are
        // scaled up, so a kernel term's fp16 low half stays a normal number
        const double amax = fmax(fabs(w0), fabs(w1)) / Wn;
        double f = (amax > 0.0 && amax < INFINITY) ? ceil(log2(amax)) : 0.0;
        f = f < -100.0 ? -100.0 : (f > 100.0 ? 100.0 : f);
        meta[meta_tc_wscale(DP) + side] = exp2(-f);
        meta[meta_tc_fold(DP) + side] = w1 >= 0.0 ? 1.0 : 0.0;
      }
    }
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
  if (A.tc16) {
    // |x'| <= c (max |x| + max |anchor|); 2^e keeps that bound <= 2^15
    __syncwarp();
    double am[2] = {0.0, 0.0};
    float *af = reinterpret_cast<float *>(meta + meta_tc_anchor(DP));
    for (int dd = lane; dd < DP; dd += 32) {
      am[0] = fmax(am[0], fabs(meta[4 + 2 * DP + dd]));
      am[1] = fmax(am[1], fabs(meta[4 + 3 * DP + dd]));
      for (int sd = 0; sd < 2; ++sd) {
        const double an = meta[4 + (2 + sd) * DP + dd];
        const float hi = (float)an;
        af[sd * 2 * DP + dd] = hi;
        af[sd * 2 * DP + DP + dd] = (float)(an - (double)hi);
      }
    }
    am[0] = warp_fmax(am[0]);
    am[1] = warp_fmax(am[1]);
    if (lane == 0) {
      const double sc = (double)pair_scale(A.scale, A.sigma_p, p);
      for (int side = 0; side < 2; ++side) {
        const double bound = sc * (cmax[side] + am[side]);
        double e = (bound > 0.0 && bound < INFINITY) ? floor(log2(32768.0 / bound)) : 0.0;
        e = e < -60.0 ? -60.0 : (e > 60.0 ? 60.0 : e);
        meta[meta_tc_cscale(DP) + side] = exp2(e);
      }
    }
  }
}

// Generic layout (D >= 4): scaled, anchored coordinates and normalised weights.
template <int NT>
__global__ void __launch_bounds__(NT) packg_kernel(PrepArgs A) {
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
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
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
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

// Tensor-core layout (ra_tc16.cuh): per 64-point tile, the fp16 hi and lo
// halves of x' 2^e in the canonical core-matrix layout (byte offset of point
// j, coordinate d: (d/8)*1024 + (j/8)*128 + (j%8)*16 + (d%8)*2), per slot
// |x'|^2, |x'|^2 - log2 a (+inf for a <= 0) and a 2^-f, and the normalised
// weights Ax / Ay.  No fp32 copy of x' (the backward packs it again from the
// points).  Masked points and the padding slots up to the tile boundary are
// zero points of zero weight.  One thread per point, walking its coordinate
// groups: a warp's stores of one group are 32 consecutive 16-byte chunks.
// V4: float4 loads of the points (D % 4 == 0, 16-byte aligned bases).
// fp16 high half of v: v with its low 13 mantissa bits cleared, exactly an
// fp16 number when |v| is in fp16's normal range; 0 below it (|v| < 2^-14:
// the low half then carries all of v).  |v| <= 2^15 by the scale choice.
__device__ __forceinline__ float tc_hi16(float v) {
  return fabsf(v) >= 6.103515625e-05f ? __uint_as_float(__float_as_uint(v) & 0xFFFFE000u) : 0.f;
}
// the fp16 bits of a value tc_hi16 returned (sign, exponent - 112, mantissa)
__device__ __forceinline__ uint32_t tc_f16_bits(float h) {
  const uint32_t b = __float_as_uint(h);
  if ((b & 0x7FFFFFFFu) == 0u) return (b >> 16) & 0x8000u;
  return ((b >> 16) & 0x8000u) | ((((b >> 13) & 0x3FFFFu) - (112u << 10)) & 0x7FFFu);
}
// two floats rounded to fp16, lo in bits 0-15
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

template <int DP, bool V4>
__global__ void __launch_bounds__(256) packtc_kernel(PrepArgs A) {
  constexpr int NG = DP / 8;     // coordinate groups per point
  constexpr int TB = DP * 128;   // bytes of a hi (or lo) tile
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
  const int D = A.D;
  for_each_chunk(M, [&](int64_t p, int side, int64_t ch, int64_t, int64_t, int64_t) {
    const Seg sg = A.seg[p];
    const int64_t s = side == 0 ? sg.xs : sg.ys;
    const int64_t count = side == 0 ? sg.xcount : sg.ycount;
    const float *pts = side == 0 ? A.x : A.y;
    const float *w = side == 0 ? A.w_x : A.w_y;
    const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
    const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
    float *Ap = side == 0 ? A.Ax : A.Ay;
    uint8_t *hp = side == 0 ? A.hx : A.hy;
    uint8_t *lp = side == 0 ? A.lx : A.ly;
    float *cp = side == 0 ? A.cx : A.cy;
    const int64_t tb = (side == 0 ? A.tbase_x : A.tbase_y)[p];
    const double *meta = A.meta + p * meta_stride(DP);
    const double Wn = meta[side];
    const float *ahi = tc_anchor(meta, DP, side), *alo = ahi + DP;
    const float sc = pair_scale(A.scale, A.sigma_p, p);
    const float cs = (float)meta[meta_tc_cscale(DP) + side];
    const float wsc = (float)meta[meta_tc_wscale(DP) + side];
    const int64_t b = ch * kChunk;
    const int64_t cend = ceil_div(count, (int64_t)kTile) * kTile;  // through the last tile
    const int64_t e = b + kChunk < cend ? b + kChunk : cend;
    for (int64_t i = b + threadIdx.x; i < e; i += 256) {
      const int64_t gi = s + i;
      const bool real = i < count;
      const bool valid = real && (mask == nullptr || mask[gi] != 0);
      const int64_t tile = tb + i / kTile;
      const int j = (int)(i % kTile);
      uint8_t *ht = hp + (size_t)tile * TB + (size_t)((j >> 3) * 128 + (j & 7) * 16);
      uint8_t *lt = lp + (size_t)tile * TB + (size_t)((j >> 3) * 128 + (j & 7) * 16);
      float sq = 0.f;
#pragma unroll 4
      for (int g = 0; g < NG; ++g) {
        float xv[8];
        if (V4 && valid && 8 * g + 8 <= D) {
          const float4 r0 = *reinterpret_cast<const float4 *>(pts + gi * D + 8 * g);
          const float4 r1 = *reinterpret_cast<const float4 *>(pts + gi * D + 8 * g + 4);
          const float rv[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
          for (int u = 0; u < 8; ++u) xv[u] = sc * ((rv[u] - ahi[8 * g + u]) - alo[8 * g + u]);
        } else {
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int d = 8 * g + u;
            xv[u] = (valid && d < D) ? sc * ((pts[gi * D + d] - ahi[d]) - alo[d]) : 0.f;
          }
        }
        uint32_t hh[4], ll[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float hv[2], lv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            hv[e] = tc_hi16(xv[2 * c + e] * cs);
            lv[e] = xv[2 * c + e] * cs - hv[e];
          }
          hh[c] = tc_f16_bits(hv[0]) | (tc_f16_bits(hv[1]) << 16);
          ll[c] = pack_half2(lv[0], lv[1]);
          sq = fmaf(xv[2 * c], xv[2 * c], sq);
          sq = fmaf(xv[2 * c + 1], xv[2 * c + 1], sq);
        }
        *reinterpret_cast<uint4 *>(ht + g * 1024) = make_uint4(hh[0], hh[1], hh[2], hh[3]);
        *reinterpret_cast<uint4 *>(lt + g * 1024) = make_uint4(ll[0], ll[1], ll[2], ll[3]);
      }
      const float a = real ? (float)((double)eff_weight(w, mask, wmode, gi) / Wn) : 0.f;
      if (real) Ap[gi] = a;
      float *cv = cp + tile * (3 * kTile);
      cv[j] = sq;
      cv[kTile + j] = a > 0.f ? sq - log2f(a) : INFINITY;
      cv[2 * kTile + j] = a * wsc;
    }
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
  const int32_t *cpair;
  unsigned *ticket;
  const int64_t *tbase_x, *tbase_y;  // [P + 1]
  int64_t max_tiles_x, max_tiles_y;
  ulonglong2 *tiles_x, *tiles_y;     // [tiles][nq = 2][64]
  float *aw_x, *aw_y;                // [tiles * 64] a~ per slot
  float *acc_x, *acc_y;              // [tiles * 64][kAcc3Stride] per-point sums, cleared
                                     // here when the tile kernel adds into them (or null)
};

// Per-side constants of the D <= 3 packing (from the pair's metadata).
struct Pack3Side {
  int64_t s, count, t0, npad;
  const float *pts, *w;
  const uint8_t *mask;
  int wmode;
  ulonglong2 *tiles;
  float *aw;
  float *acc;  // the slots' per-point sums, zeroed with the packing (or null)
  double Wm;  // a~ = w' / Wm
  bool fold, uni;
  float pad, ax, ay, az, scale;
};

__device__ __forceinline__ Pack3Side pack3_side(const PackArgs &A, int64_t p, int side,
                                                const Seg &sg) {
  Pack3Side S;
  S.s = side == 0 ? sg.xs : sg.ys;
  S.count = side == 0 ? sg.xcount : sg.ycount;
  S.t0 = (side == 0 ? A.tbase_x : A.tbase_y)[p];
  const int64_t t1 = (side == 0 ? A.tbase_x : A.tbase_y)[p + 1];
  // the tiles the kernels read: ceil(count / 64), within the room reserved
  const int64_t nt = ceil_div(S.count, (int64_t)kTile);
  S.npad = (nt < t1 - S.t0 ? nt : t1 - S.t0) * kTile;
  S.pts = side == 0 ? A.x : A.y;
  S.w = side == 0 ? A.w_x : A.w_y;
  S.mask = side == 0 ? A.mask_x : A.mask_y;
  S.wmode = side == 0 ? A.wmode_x : A.wmode_y;
  S.tiles = side == 0 ? A.tiles_x : A.tiles_y;
  S.aw = side == 0 ? A.aw_x : A.aw_y;
  S.acc = side == 0 ? A.acc_x : A.acc_y;
  const double *meta = A.meta + p * meta_stride(3);
  S.Wm = meta[side] * meta[meta_wscale(3) + side];
  S.fold = meta[meta_fold(3) + side] != 0.0;
  S.uni = meta[meta_fold(3) + side] == 2.0;
  S.pad = S.uni ? 1e18f : 0.f;
  S.ax = (float)meta[4 + (2 + side) * 3 + 0];
  S.ay = (float)meta[4 + (2 + side) * 3 + 1];
  S.az = (float)meta[4 + (2 + side) * 3 + 2];
  S.scale = pair_scale(A.scale, A.sigma_p, p);
  return S;
}

// Slot i (< S.npad) of a side's tiles: a point (i < count) or padding.
__device__ __forceinline__ void pack3_slot(const PackArgs &A, const Pack3Side &S, int64_t i) {
  const int D = A.D;
  float c0 = S.pad, c1 = S.pad, c2 = S.pad, a = 0.f, v = S.fold ? INFINITY : 0.f;
  if (i < S.count) {
    const int64_t g = S.s + i;
    const double at = S.uni ? 1.0 : (double)eff_weight(S.w, S.mask, S.wmode, g) / S.Wm;
    a = (float)at;
    c1 = c2 = 0.f;
    // folded: a~ in [0, 1]; a zero weight becomes 2^-64, which leaves the
    // other points' sums unchanged to 5e-20 and keeps the point's own
    // row sums (its weight gradient) finite
    v = S.fold ? (at >= 1.0 ? 0.f : at > 0x1p-64 ? (float)-log2(at) : 64.f) : a;
    c0 = S.scale * (S.pts[g * D + 0] - S.ax);
    if (D > 1) c1 = S.scale * (S.pts[g * D + 1] - S.ay);
    if (D > 2) c2 = S.scale * (S.pts[g * D + 2] - S.az);
  }
  const int64_t t = S.t0 + i / kTile;
  ulonglong2 *tp = S.tiles + t * (int64_t)(A.nq * kTile) + (i % kTile);
  tp[0] = make_ulonglong2(pk2u(c0, c0), pk2u(c1, c1));
  tp[kTile] = make_ulonglong2(pk2u(c2, c2), pk2u(v, v));
  S.aw[t * (int64_t)kTile + (i % kTile)] = a;
  if (S.acc != nullptr) {
    // the slot's sums start at zero: the tile kernel adds its column sums in
    float4 *r = reinterpret_cast<float4 *>(S.acc + (t * (int64_t)kTile + (i % kTile)) * kAcc3Stride);
    r[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    r[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

template <int NT>
__global__ void __launch_bounds__(NT) pack3_kernel(PackArgs A) {
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
  for_each_chunk(M, [&](int64_t p, int side, int64_t c, int64_t, int64_t, int64_t) {
    const Seg sg = A.seg[p];
    if (small_pair(sg)) return;  // packed by prep3_kernel
    const Pack3Side S = pack3_side(A, p, side, sg);
    const int64_t tmax = side == 0 ? A.max_tiles_x : A.max_tiles_y;
    const int64_t b = c * kChunk, e = b + kChunk < S.npad ? b + kChunk : S.npad;
    for (int64_t i = b + threadIdx.x; i < e; i += NT) {
      if (S.t0 + i / kTile >= tmax) break;  // malformed ptr overflowing the bound (flagged)
      pack3_slot(A, S, i);
    }
  });
}

// Error-free accumulation in float32 (Knuth's TwoSum, the running error kept
// in a second float): a double-float sum of a few thousand floats, free of
// float-to-double conversions per point, which run on the SM's narrow
// conversion pipe.
struct FSum {
  float hi = 0.f, lo = 0.f;
  __device__ __forceinline__ void add(float v) {
    const float s = hi + v, bp = s - hi;
    lo += (hi - (s - bp)) + (v - bp);
    hi = s;
  }
  // adds the exact product a * b (TwoProduct by FMA)
  __device__ __forceinline__ void add_prod(float a, float b) {
    const float q = a * b;
    add(q);
    lo += fmaf(a, b, -q);
  }
  __device__ __forceinline__ double value() const { return (double)hi + (double)lo; }
};

// D <= 3, pairs with at most kSmallPts points per side (small_pair): one CTA
// per pair does what stats3_kernel, meta_kernel and pack3_kernel do for the
// large pairs -- the sums of both sides, the metadata, the packing -- so the
// points are read from DRAM once (the packing pass re-reads them from cache).
template <int NT>
__global__ void __launch_bounds__(NT) prep3_kernel(PrepArgs A, PackArgs K) {
  __shared__ double sh[(NT / 32) * 8];
  __shared__ long long shl[NT / 32];
  __shared__ float shm[NT / 32][2];
  __shared__ double tot[2][12];  // per side: W, nv, sum w'p (3), sum p (3), last, wmax, nwmin
  __shared__ unsigned pt_slot[2];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int D = A.D;
  unsigned pt_nxt = 0;
  int pt_k = 0;
  for (int64_t p = pair_ticket_first(A.pair_ticket, pt_slot); p < A.P;
       p = pair_ticket_next(pt_slot, ++pt_k, pt_nxt)) {
    pt_nxt = pair_ticket_take(A.pair_ticket);
    Seg sg = A.seg[p];
    if (!small_pair(sg)) continue;
    for (int side = 0; side < 2; ++side) {
      const float *pts = side == 0 ? A.x : A.y;
      const float *w = side == 0 ? A.w_x : A.w_y;
      const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
      const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
      const int64_t s = side == 0 ? sg.xs : sg.ys;
      const int64_t span = side == 0 ? sg.xspan : sg.yspan;
      FSum W, cs[3], ps[3];
      int nv = 0;
      long long last = -1;
      float wmax = -INFINITY, nwmin = -INFINITY;
      for (int64_t i = tid; i < span; i += NT) {
        const int64_t g = s + i;
        const float wi = eff_weight(w, mask, wmode, g);
        const bool valid = mask == nullptr || mask[g] != 0;
        W.add(wi);
        wmax = fmaxf(wmax, wi);
        nwmin = fmaxf(nwmin, -wi);
#pragma unroll
        for (int d = 0; d < 3; ++d) {
          if (d < D) {
            const float pv = pts[g * D + d];
            cs[d].add_prod(wi, pv);
            if (valid) ps[d].add(pv);
          }
        }
        if (valid) {
          ++nv;
          last = i;
        }
      }
      double vals[8] = {W.value(), (double)nv, cs[0].value(), cs[1].value(), cs[2].value(),
                        ps[0].value(), ps[1].value(), ps[2].value()};
      last = warp_max(last);
      float wm = wmax, nw = nwmin;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        wm = fmaxf(wm, __shfl_xor_sync(kFull, wm, o));
        nw = fmaxf(nw, __shfl_xor_sync(kFull, nw, o));
      }
      if (lane == 0) {
        shl[wid] = last;
        shm[wid][0] = wm;
        shm[wid][1] = nw;
      }
      block_sum_n<8>(vals, sh);  // its first barrier also publishes shl and shm
      if (tid == 0) {
        long long lst = -1;
        float mx = -INFINITY, nmn = -INFINITY;
        for (int k = 0; k < NT / 32; ++k) {
          lst = shl[k] > lst ? shl[k] : lst;
          mx = fmaxf(mx, shm[k][0]);
          nmn = fmaxf(nmn, shm[k][1]);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) tot[side][k] = vals[k];
        tot[side][8] = (double)lst;
        tot[side][9] = (double)mx;
        tot[side][10] = (double)nmn;
      }
      // shl / shm are rewritten by the next side after block_sum_n's trailing barrier
    }
    __syncthreads();
    // ---- metadata (meta_kernel's semantics), one thread -------------------
    if (tid == 0) {
      double *meta = A.meta + p * meta_stride(3);
      if (A.sigma_p != nullptr && !(A.sigma_p[p] > 0.0)) atomicOr(A.err, (int)kErrSigma);
      int64_t count_x = 0;
      for (int side = 0; side < 2; ++side) {
        const double *t = tot[side];
        const double W = t[0], nv = t[1];
        const int64_t span = side == 0 ? sg.xspan : sg.yspan;
        const int64_t count = A.layout == 0 ? span : (int64_t)t[8] + 1;
        const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
        double Wn, m, fold;
        bool werr;
        side_normaliser(wmode, W, nv, count, A.allow_fold != 0, t[9], t[10], Wn, m, fold, werr);
        if (werr) atomicOr(A.err, (int)kErrWeightSum);
        meta[side] = Wn;
        meta[2 + side] = W;
        meta[meta_wscale(3) + side] = m;
        meta[meta_fold(3) + side] = fold;
        if (side == 0) {
          sg.xcount = count;
          count_x = count;
        } else {
          sg.ycount = count;
        }
        for (int dd = 0; dd < 3; ++dd) {
          const double mu = dd < D ? t[2 + dd] / Wn : 0.0;
          const double mean = (dd < D && nv > 0) ? t[5 + dd] / nv : 0.0;
          meta[4 + side * 3 + dd] = mu;
          if (side == 0) {
            meta[4 + 6 + dd] = mean;  // provisional: replaced by the anchor below
          } else {
            double ax, ay;
            if (A.center) {
              ax = meta[4 + dd];
              ay = mu;
            } else {
              ax = count_x > 0 ? meta[4 + 6 + dd] : mean;
              ay = ax;
            }
            meta[4 + 6 + dd] = ax;
            meta[4 + 9 + dd] = ay;
          }
        }
      }
      A.seg[p].xcount = sg.xcount;
      A.seg[p].ycount = sg.ycount;
    }
    __syncthreads();
    // ---- packing: the tiles of both sides (points re-read from cache) -----
    sg = A.seg[p];
    for (int side = 0; side < 2; ++side) {
      const Pack3Side S = pack3_side(K, p, side, sg);
      for (int64_t i = tid; i < S.npad; i += NT) pack3_slot(K, S, i);
    }
    __syncthreads();  // tot is rewritten by the next pair
  }
}

}  // namespace ra
