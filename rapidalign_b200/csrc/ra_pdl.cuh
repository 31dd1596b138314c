// ra_pdl.cuh -- the pairwise-distance spectrum loss (rapidalign/algorithms.py:
// 19-90): per group g of points, the distances of all pairs i < j of the
// source group and of the target group, each sorted ascending, the shorter
// list padded with zeros at its end, and loss_g = mean((s_k - t_k)^2) over
// the longer length L_g (0 / 0 = NaN for two groups of < 2 points, as
// torch's mean of an empty tensor).
//
// B200 layout: one flat array of pair distances per side, the pairs of group
// g at [poff[g], poff[g+1]) in row-major upper-triangle order (pair (i, j)
// at i n - i (i + 1) / 2 + j - i - 1), written by a grid-stride kernel
// (coalesced stores, HBM-bound); a segmented radix sort of (distance, pair)
// per group (CUB's DeviceSegmentedSort, header-only); one CTA per group for
// the loss (fp64, fixed order).  The backward scatters d loss / d s_k to the
// pair's two points through the sorted pair ids: dL/dp_i += g (p_i - p_j) / d,
// dL/dp_j -= the same (fp32 atomics), 0 for d = 0 like torch's norm.
// Points are addressed through an optional permutation (perm[ptr[g] + i]), so
// groups given by unsorted batch ids need no reordering copy.
#pragma once

#include <cub/device/device_segmented_sort.cuh>

#include "ra_common.cuh"

namespace ra {

struct PdlSide {
  const float *pts;      // [N, D]
  const int64_t *perm;   // [N] point of grouped position, or null (identity)
  const int64_t *ptr;    // [G + 1] grouped positions of each group
  const int64_t *poff;   // [G + 1] pair offsets
  int64_t pairs;
  float *keys;           // [pairs] distances (sorted by the forward)
  uint32_t *vals;        // [pairs] (i << 16) | j
};

__device__ __forceinline__ int64_t pdl_group_of(const int64_t *poff, int64_t G, int64_t k) {
  int64_t lo = 0, hi = G;  // poff[lo] <= k < poff[hi]
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (poff[mid] <= k) lo = mid;
    else hi = mid;
  }
  return lo;
}

// Pair k of a group of n points in row-major upper-triangle order -> (i, j).
__device__ __forceinline__ void pdl_decode(int64_t k, int64_t n, int64_t &i, int64_t &j) {
  // rows before i hold off(i) = i n - i (i + 1) / 2 pairs: invert, then fix
  const double b = 2.0 * (double)n - 1.0;
  int64_t r = (int64_t)((b - sqrt(b * b - 8.0 * (double)k)) * 0.5);
  if (r < 0) r = 0;
  if (r > n - 2) r = n - 2;
  while (r > 0 && r * n - r * (r + 1) / 2 > k) --r;
  while (r + 1 <= n - 2 && (r + 1) * n - (r + 1) * (r + 2) / 2 <= k) ++r;
  i = r;
  j = k - (r * n - r * (r + 1) / 2) + r + 1;
}

__global__ void pdl_dist_kernel(PdlSide S, int64_t G, int D) {
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < S.pairs;
       k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t g = pdl_group_of(S.poff, G, k);
    const int64_t n = S.ptr[g + 1] - S.ptr[g];
    int64_t i, j;
    pdl_decode(k - S.poff[g], n, i, j);
    const int64_t a = S.ptr[g] + i, b = S.ptr[g] + j;
    const int64_t pa = S.perm ? S.perm[a] : a, pb = S.perm ? S.perm[b] : b;
    float r2 = 0.f;
    for (int d = 0; d < D; ++d) {
      const float t = S.pts[pa * D + d] - S.pts[pb * D + d];
      r2 = fmaf(t, t, r2);
    }
    S.keys[k] = sqrtf(r2);
    S.vals[k] = ((uint32_t)i << 16) | (uint32_t)j;
  }
}

// One CTA per group: loss_g = sum_k (s_k - t_k)^2 / L_g over the sorted lists.
__global__ void __launch_bounds__(256) pdl_loss_kernel(PdlSide Sx, PdlSide Sy, int64_t G,
                                                       double *loss) {
  __shared__ double sh[256 / 32];
  const int64_t g = blockIdx.x;
  const int64_t ns = Sx.poff[g + 1] - Sx.poff[g], nt = Sy.poff[g + 1] - Sy.poff[g];
  const int64_t L = ns > nt ? ns : nt;
  const float *s = Sx.keys + Sx.poff[g], *t = Sy.keys + Sy.poff[g];
  double acc = 0.0;
  for (int64_t k = threadIdx.x; k < L; k += blockDim.x) {
    const double dv = (double)(k < ns ? s[k] : 0.f) - (double)(k < nt ? t[k] : 0.f);
    acc += dv * dv;
  }
  acc = block_sum(acc, sh);
  if (threadIdx.x == 0) loss[g] = acc / (double)L;  // 0 / 0 = NaN for L = 0
}

// Gradients of sum_g up_g loss_g with respect to the points of side S (O is
// the other side): d loss_g / d (own k-th distance) = 2 (own_k - other_k) / L_g.
__global__ void pdl_grad_kernel(PdlSide S, PdlSide O, int64_t G, int D, const double *up,
                                float *grad) {
  for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < S.pairs;
       k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t g = pdl_group_of(S.poff, G, k);
    const int64_t kk = k - S.poff[g];
    const int64_t ns = S.poff[g + 1] - S.poff[g], no = O.poff[g + 1] - O.poff[g];
    const int64_t L = ns > no ? ns : no;
    const float sk = S.keys[k];
    const float ok = kk < no ? O.keys[O.poff[g] + kk] : 0.f;
    const double gd = 2.0 * ((double)sk - (double)ok) / (double)L * up[g];
    if (!(sk > 0.f)) continue;  // zero distance: zero gradient (torch's norm)
    const uint32_t v = S.vals[k];
    const int64_t a = S.ptr[g] + (v >> 16), b = S.ptr[g] + (v & 0xFFFFu);
    const int64_t pa = S.perm ? S.perm[a] : a, pb = S.perm ? S.perm[b] : b;
    const float coef = (float)(gd / (double)sk);
    for (int d = 0; d < D; ++d) {
      const float vec = coef * (S.pts[pa * D + d] - S.pts[pb * D + d]);
      atomicAdd(grad + pa * D + d, vec);
      atomicAdd(grad + pb * D + d, -vec);
    }
  }
}

}  // namespace ra
