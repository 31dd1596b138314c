// ra_prep.cuh -- per-pair preparation: segment bounds, weight normalisation,
// weighted centroids and packing of the points into the layouts the tile
// kernels read.  One CTA per pair.
//
// Semantics follow rapidalign/kde.py:
//   ptr checks            kde.py:124-156 (plus a monotonicity check)
//   weight normalisation  kde.py:20-27 (single), 169-199 (ragged),
//                         115-121 (dense, clamped), 183-188 (uniform)
//   centering             kde.py:77-81, 202-208, 246-253
// Distances are translation invariant, so without centering both clouds are
// still shifted by one common anchor (the x centroid); this keeps the packed
// coordinates small and changes no result.
#pragma once

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
__host__ __device__ __forceinline__ int meta_stride(int DP) { return 4 + 4 * DP; }

struct PrepArgs {
  int64_t P;
  int D, DP;     // DP: 3 for the D <= 3 path, else the padded generic width
  int layout;    // 0 ragged, 1 dense
  int wmode_x, wmode_y, center;
  int packed3;   // 1: write the D <= 3 tile layout, 0: the generic layout
  int64_t num_x, num_y, nmax_x, nmax_y;
  float scale;   // sqrt(log2(e) / (2 sigma^2)): packed coords are scale * (p - anchor)
  const float *x, *y, *w_x, *w_y;
  const int64_t *ptr_x, *ptr_y;
  const uint8_t *mask_x, *mask_y;
  Seg *seg;
  double *meta;
  int *err;
  // generic layout (D >= 4): coords [num * DP] (zero padded) and weights [num]
  float *Gx, *Gy, *Ax, *Ay;
};

// Effective (masked, raw) weight of point i.
__device__ __forceinline__ float eff_weight(const float *w, const uint8_t *mask, int wmode,
                                            int64_t i) {
  float v = (wmode == 3 || w == nullptr) ? 1.0f : w[i];
  if (mask != nullptr && mask[i] == 0) v = 0.0f;
  return v;
}

// Reduction width: power of two >= D (at least 4).
__device__ __forceinline__ int red_width(int D) {
  int r = 4;
  while (r < D) r <<= 1;
  return r;
}

template <int NT>
__device__ void prep_side(const PrepArgs &A, int64_t p, int side, double *sh, int64_t *shl) {
  const int tid = threadIdx.x;
  const int D = A.D, DP = A.DP;
  const float *pts = side == 0 ? A.x : A.y;
  const float *w = side == 0 ? A.w_x : A.w_y;
  const uint8_t *mask = side == 0 ? A.mask_x : A.mask_y;
  const int wmode = side == 0 ? A.wmode_x : A.wmode_y;
  const int64_t num = side == 0 ? A.num_x : A.num_y;
  const int64_t *ptr = side == 0 ? A.ptr_x : A.ptr_y;
  const int64_t nmax = side == 0 ? A.nmax_x : A.nmax_y;
  double *meta = A.meta + p * meta_stride(DP);
  Seg &sg = A.seg[p];

  // ---- segment bounds ------------------------------------------------------
  int64_t s, span;
  if (A.layout == 0) {
    int64_t a0 = ptr[p], a1 = ptr[p + 1];
    if (tid == 0) {
      int e = 0;
      if (p == 0 && a0 != 0) e |= kErrPtrStart;
      if (p == A.P - 1 && a1 != num) e |= kErrPtrEnd;
      if (a1 < a0) e |= kErrPtrOrder;
      if (e) atomicOr(A.err, e);
    }
    // clamp so that a malformed ptr can never send a kernel out of bounds
    a0 = a0 < 0 ? 0 : (a0 > num ? num : a0);
    a1 = a1 < a0 ? a0 : (a1 > num ? num : a1);
    s = a0;
    span = a1 - a0;
  } else {
    s = p * nmax;
    span = nmax;
  }

  // ---- pass 1: weight sum, weighted coordinate sums, last valid index -------
  const int RW = red_width(D);
  const int lanes = NT / RW;  // point lanes
  const int d = tid % RW, pl = tid / RW;
  double acc = 0.0, accu = 0.0, wsum = 0.0;
  int64_t last = -1;
  int64_t nvalid = 0;
  for (int64_t i = pl; i < span; i += lanes) {
    const int64_t g = s + i;
    const float wi = eff_weight(w, mask, wmode, g);
    const bool valid_pt = mask == nullptr || mask[g] != 0;
    if (d < D) {
      const double v = (double)pts[g * D + d];
      acc += (double)wi * v;
      if (valid_pt) accu += v;
    }
    if (d == 0) {
      wsum += (double)wi;
      const bool valid = mask == nullptr || mask[g] != 0;
      if (valid) {
        last = i;
        ++nvalid;
      }
    }
  }
  sh[tid] = acc;
  __syncthreads();
  double coord_sum = 0.0;
  if (tid < RW)
    for (int l = 0; l < lanes; ++l) coord_sum += sh[l * RW + tid];
  __syncthreads();
  sh[tid] = accu;
  __syncthreads();
  double plain_sum = 0.0;  // unweighted sum of the valid points (anchor)
  if (tid < RW)
    for (int l = 0; l < lanes; ++l) plain_sum += sh[l * RW + tid];
  __syncthreads();
  sh[tid] = wsum;
  shl[tid] = last;
  shl[NT + tid] = nvalid;
  __syncthreads();
  if (tid == 0) {
    double W = 0.0;
    int64_t lst = -1, nv = 0;
    for (int l = 0; l < lanes; ++l) {
      W += sh[l * RW];
      lst = shl[l * RW] > lst ? shl[l * RW] : lst;
      nv += shl[NT + l * RW];
    }
    const int64_t count = A.layout == 0 ? span : lst + 1;
    double Wn;
    if (wmode == 0) {
      Wn = 1.0;  // raw weights
    } else if (wmode == 3) {
      Wn = nv > 0 ? (double)nv : 1.0;  // uniform 1/count
    } else if (wmode == 2) {
      Wn = W > 1e-8 ? W : 1e-8;  // clamp_min(1e-8)
    } else {
      Wn = W;
      if (count > 0 && !(W > 0.0) && !(W != W)) atomicOr(A.err, (int)kErrWeightSum);
      if (!(W > 0.0)) Wn = 1.0;  // keep the kernels finite; the error is reported
    }
    meta[side] = Wn;
    meta[2 + side] = W;
    if (side == 0) {
      sg.xs = s;
      sg.xspan = span;
      sg.xcount = count;
    } else {
      sg.ys = s;
      sg.yspan = span;
      sg.ycount = count;
    }
    sh[NT] = Wn;
    shl[0] = nv;
  }
  __syncthreads();
  const double Wn = sh[NT];
  const int64_t nvalid_all = shl[0];
  // centroid mu = sum_i a_i p_i = sum_i w'_i p_i / Wn
  if (tid < DP) {
    const double mu = tid < D ? coord_sum / Wn : 0.0;
    meta[4 + side * DP + tid] = mu;
  }
  __syncthreads();
  // anchors.  Centering: each cloud is shifted by its weighted centroid (the
  // semantics).  Otherwise both clouds share one anchor, the unweighted mean
  // of the valid x points (of the y points when x has none): distances do not
  // change, and the packed coordinates stay as small as the clouds themselves
  // whatever the weights are (raw weights may be negative).
  if (tid < DP) {
    const double mean = (tid < D && nvalid_all > 0) ? plain_sum / (double)nvalid_all : 0.0;
    double anc;
    if (A.center) {
      anc = meta[4 + side * DP + tid];
    } else if (side == 0) {
      anc = mean;
    } else {
      anc = sg.xcount > 0 ? meta[4 + 2 * DP + tid] : mean;
    }
    meta[4 + (2 + side) * DP + tid] = anc;
    sh[NT + 1 + tid] = anc;
  }
  __syncthreads();

  // ---- pass 2 (generic layout only): pack ---------------------------------
  // (the D <= 3 tile layout is written by pack3_kernel once the tile bases
  // of all pairs are known)
  const int64_t count = side == 0 ? sg.xcount : sg.ycount;
  const float scale = A.scale;
  if (!A.packed3) {
    float *Gp = side == 0 ? A.Gx : A.Gy;
    float *Ap = side == 0 ? A.Ax : A.Ay;
    for (int64_t i = pl; i < count; i += lanes) {
      const int64_t g = s + i;
      if (d < DP) {
        float v = 0.f;
        if (d < D) v = scale * (float)((double)pts[g * D + d] - sh[NT + 1 + d]);
        Gp[g * DP + d] = v;
      }
      if (d == 0) {
        const float wi = eff_weight(w, mask, wmode, g);
        Ap[g] = (float)((double)wi / Wn);
      }
    }
  }
  __syncthreads();
}

template <int NT>
__global__ void __launch_bounds__(NT) prep_kernel(PrepArgs A) {
  // sh: NT doubles for reductions + 1 + DP anchors; shl: 2*NT ints
  extern __shared__ double smem[];
  double *sh = smem;
  int64_t *shl = (int64_t *)(smem + NT + 1 + 256);
  const int64_t p = blockIdx.x;
  if (p >= A.P) return;
  prep_side<NT>(A, p, 0, sh, shl);
  prep_side<NT>(A, p, 1, sh, shl);
}

// ---------------------------------------------------------------------------
// D <= 3 tile layout.  Each cloud is cut into 64-point tiles, zero-weight
// padded; pair p's x tiles start at tile tbase_x[p] (exclusive scan of
// ceil(count / 64)).  A tile stores two arrays of 64 duplicated pairs
// (16 bytes per point each):  {x', x', y', y'}  and  {z', z', w, w}
// so one column feeds packed f32x2 arithmetic against two rows, and a warp
// reads any column of a tile at an immediate offset from the tile base.
// ---------------------------------------------------------------------------
struct PackArgs {
  int64_t P;
  int D, nq;
  float scale;
  const float *x, *y, *w_x, *w_y;
  const uint8_t *mask_x, *mask_y;
  int wmode_x, wmode_y;
  const Seg *seg;
  const double *meta;
  const int64_t *tbase_x, *tbase_y;  // [P + 1]
  int64_t max_tiles_x, max_tiles_y;
  ulonglong2 *tiles_x, *tiles_y;     // [tiles][nq = 2][64]
};

template <int NT>
__global__ void __launch_bounds__(NT) pack3_kernel(PackArgs A) {
  const int64_t p = blockIdx.x >> 1;
  const int side = blockIdx.x & 1;
  if (p >= A.P) return;
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
  const double *meta = A.meta + p * meta_stride(3);
  const double Wn = meta[side];
  const float ax = (float)meta[4 + (2 + side) * 3 + 0];
  const float ay = (float)meta[4 + (2 + side) * 3 + 1];
  const float az = (float)meta[4 + (2 + side) * 3 + 2];
  const float scale = A.scale;
  const int nq = A.nq;
  const int64_t npad = (t1 - t0) * kTile;
  for (int64_t i = threadIdx.x; i < npad; i += NT) {
    const int64_t t = t0 + i / kTile;
    if (t >= tmax) break;  // malformed ptr overflowing the bound (error already flagged)
    float c0 = 0.f, c1 = 0.f, c2 = 0.f, a = 0.f;
    if (i < count) {
      const int64_t g = s + i;
      a = (float)((double)eff_weight(w, mask, wmode, g) / Wn);
      c0 = scale * (pts[g * D + 0] - ax);
      if (D > 1) c1 = scale * (pts[g * D + 1] - ay);
      if (D > 2) c2 = scale * (pts[g * D + 2] - az);
    }
    ulonglong2 *tp = tiles + t * (int64_t)(nq * kTile) + (i % kTile);
    tp[0] = make_ulonglong2(pk2u(c0, c0), pk2u(c1, c1));
    tp[kTile] = make_ulonglong2(pk2u(c2, c2), pk2u(a, a));
  }
}


}  // namespace ra
