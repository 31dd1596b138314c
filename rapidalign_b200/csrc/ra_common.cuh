// ra_common.cuh -- shared device helpers and internal data structures of the
// B200 KDE/MMD library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace ra {

constexpr unsigned kFull = 0xffffffffu;

// ---------------------------------------------------------------------------
// Packed-FP32 arithmetic.  sm_100 issues two fp32 lanes per instruction with
// the .f32x2 forms; the FP32 pipe throughput is unchanged, the issue-slot cost
// halves.  A "pair" is a 64-bit register holding {lo, hi}.
// ---------------------------------------------------------------------------
typedef unsigned long long f2_t;

__device__ __forceinline__ f2_t pk(float lo, float hi) {
  f2_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk(f2_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long pk2u(float lo, float hi) {
  return ((unsigned long long)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float lo_of(f2_t v) {
  float lo, hi;
  upk(v, lo, hi);
  return lo;
}
__device__ __forceinline__ float hi_of(f2_t v) {
  float lo, hi;
  upk(v, lo, hi);
  return hi;
}
__device__ __forceinline__ f2_t add2(f2_t a, f2_t b) {
  f2_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2_t sub2(f2_t a, f2_t b) {
  f2_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2_t mul2(f2_t a, f2_t b) {
  f2_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2_t fma2(f2_t a, f2_t b, f2_t c) {
  f2_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Coordinate pre-scale for bandwidth sigma: packed coordinates are
// c (p - anchor) with c^2 = log2(e) / (2 sigma^2), so that
// exp(-|u - v|^2 / (2 sigma^2)) = 2^(-|c u - c v|^2).  The same float on the
// host and on the device (sqrt is correctly rounded on both).
__host__ __device__ __forceinline__ float scale_of_sigma(double sigma) {
  return (float)sqrt(1.4426950408889634 / (2.0 * sigma * sigma));
}

// 2^x on the SFU (MUFU.EX2), flush-to-zero: inputs below -126 give 0, which
// is the same as the true value to within 1.2e-38.
__device__ __forceinline__ float ex2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Vector reduction into global memory, performed at L2 (sm_90+).
__device__ __forceinline__ void red_add_v4(float *addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// Block-wide sum of one double (all threads get the result).  `sh` must hold
// blockDim.x / 32 doubles; contains a __syncthreads on both sides.
__device__ __forceinline__ double block_sum(double v, double *sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < nw; ++w) t += sh[w];  // fixed order: deterministic
  return t;
}

// Block-wide sums of N doubles at once (all threads get the results): a
// shuffle tree inside each warp, then the warps in order -- deterministic.
// `sh` must hold (blockDim.x / 32) * N doubles; two __syncthreads.
template <int N>
__device__ __forceinline__ void block_sum_n(double (&v)[N], double *sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int k = 0; k < N; ++k) v[k] = warp_sum(v[k]);
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < N; ++k) sh[wid * N + k] = v[k];
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < N; ++k) {
    double t = 0.0;
    for (int w = 0; w < nw; ++w) t += sh[w * N + k];
    v[k] = t;
  }
  __syncthreads();
}

__device__ __forceinline__ long long warp_max(long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const long long u = __shfl_xor_sync(kFull, v, o);
    v = u > v ? u : v;
  }
  return v;
}
__device__ __forceinline__ double warp_fmax(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(kFull, v, o));
  return v;
}
__device__ __forceinline__ float warp_fmaxf(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// Internal data structures (live in the caller's workspace).
// ---------------------------------------------------------------------------

// Error word bits (device-detected data errors), see ra_status in the header.
enum : int {
  kErrPtrStart = 1,
  kErrPtrEnd = 2,
  kErrPtrOrder = 4,
  kErrWeightSum = 8,
  kErrTimeout = 16,  // a bounded device-side wait expired (tensor-core kernels, ring passes)
  kErrSigma = 32,    // a per-pair bandwidth is not > 0
};

// Per pair: where its points live and how many of them the kernels visit.
// For ragged inputs span == count.  For dense inputs span == Nmax and count is
// 1 + the last valid (mask != 0) index, so the padded tail is never computed.
struct Seg {
  int64_t xs, xspan, xcount;
  int64_t ys, yspan, ycount;
};

// floats per point in the D <= 3 accumulator record: per block (self, then
// cross) the sums (s, G0, G1, G2)
constexpr int kAcc3Stride = 8;
constexpr int kAcc3Block = 4;

// Tile geometry of the D <= 3 kernel.
constexpr int kTile = 64;          // rows per warp item and columns per tile
constexpr int kSplitMax = 16;      // max column splits of one row tile
constexpr int kSplitMinTiles = 64; // a split covers at least this many col tiles

// Per-point record of the generic (D >= 4) layout, in floats: T_self[DP],
// T_cross[DP], s_self, s_cross, 2 pad.  The T segments start 16-byte
// aligned, so kernels write and read them as float4.
__host__ __device__ constexpr int gen_acc_stride(int DP) { return 2 * DP + 4; }

// Tile geometry of the generic-D kernel (one thread per row).
constexpr int kGenRows = 128;
constexpr int kGenCols = 32;

__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) {
  return (a + b - 1) / b;
}

// Column splits of a row tile whose column range has nTc tiles.
__host__ __device__ __forceinline__ int64_t splits_for(int64_t nTc) {
  int64_t s = ceil_div(nTc, (int64_t)kSplitMinTiles);
  if (s < 1) s = 1;
  return s > kSplitMax ? kSplitMax : s;
}

// Work item of the D <= 3 kernel: (pair, block, row tile, split).
//   block 0: rows x, cols y  (cross, Kxy)
//   block 1: rows x, cols x  (self, symmetric, Kxx)
//   block 2: rows y, cols y  (self, symmetric, Kyy)
// Work item of the generic kernel: (pair, orientation, row tile, 0) with
//   orientation 0: x vs y, 1: x vs x, 2: y vs y, 3: y vs x.
struct Item {
  int pair, block, tile, split;
};

}  // namespace ra
