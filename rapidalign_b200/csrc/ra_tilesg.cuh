// ra_tilesg.cuh -- generic-dimension kernel (D >= 4, DP = D rounded up to a
// power of two).  One thread per row, 128 rows per CTA, columns staged through
// shared memory 32 at a time.  Every block is visited in both orientations
// (x-y, x-x, y-y, y-x), so each point's row sums are complete when its CTA
// finishes and are written without atomics.  This path covers any D; the
// D <= 3 point-cloud path is ra_tiles3.cuh.
//
// The row sums are kept in folded form, G_i = x'_i s_i - T_i with
// T_i = sum_j w_j k_ij y'_j.  In a self block the diagonal term (j == i,
// k_ii = 1) would put w_i x'_i into T_i and w_i into s_i, to cancel in G_i only
// up to fp32 rounding -- an error far above the true G_i when the kernel is
// narrow.  The stored sums therefore leave the diagonal out; it re-enters
// exactly: in the pair sum here and in dL/da in the epilogue.
#pragma once

#include "ra_common.cuh"

namespace ra {

struct TilesGArgs {
  const Item *items;
  const int64_t *n_items;
  const Seg *seg;
  const float *Gx, *Gy;  // [num * DP] packed coordinates
  const float *Ax, *Ay;  // [num] normalised weights
  float *accX, *accY;    // [num][2 + 2*DP]: self (s, T[DP]), cross (s, T[DP])
  double *itemK, *itemS;
  int need_rows;         // 1: write the per-point sums (backward requested)
  int shard_index, shard_count;  // evaluate only items shard_index + k * shard_count
  int *err;                      // error word (the tensor-core path's wait limits)
  unsigned spin_limit;           // tensor-core path: polls of one wait before giving up
  int no_mma;                    // test hook: the tensor-core path issues no MMA at all
};

// One staged column tile against this thread's row: st += sum w, T += sum w y'
// (and sgt += sum w r^2).  DIAG: the term in column `diag` is left out.
template <int DP, int MODE, bool DIAG>
__device__ __forceinline__ void gen_cols(const float *ycol, const float *bcol,
                                         const float (&xr)[DP], float (&T)[DP], float &st,
                                         float &sgt, int diag) {
  constexpr bool SIG = MODE == 2;
#pragma unroll 1
  for (int jj = 0; jj < kGenCols; ++jj) {
    const float *yj = ycol + jj * DP;
    float r2 = 0.f;
#pragma unroll
    for (int d = 0; d < DP; ++d) {
      const float t = xr[d] - yj[d];
      r2 = fmaf(t, t, r2);
    }
    float w = bcol[jj] * ex2(-r2);
    if (DIAG && jj == diag) w = 0.f;
    st += w;
    if (SIG) sgt = fmaf(w, r2, sgt);
    if (MODE >= 1) {
#pragma unroll
      for (int d = 0; d < DP; ++d) T[d] = fmaf(w, yj[d], T[d]);
    }
  }
}

template <int DP, int MODE>
__global__ void __launch_bounds__(kGenRows) tilesg_kernel(TilesGArgs A) {
  constexpr bool SIG = MODE == 2;
  __shared__ float ycol[kGenCols * DP];
  __shared__ float bcol[kGenCols];
  __shared__ double red[kGenRows / 32 * 2];
  const int64_t it = blockIdx.x;
  if (it >= *A.n_items || it % A.shard_count != A.shard_index) return;
  const Item item = A.items[it];
  const Seg sg = A.seg[item.pair];
  const int o = item.block;  // 0: x-y, 1: x-x, 2: y-y, 3: y-x
  const bool rows_x = (o == 0 || o == 1);
  const bool cols_x = (o == 1 || o == 3);
  const int64_t rbase = rows_x ? sg.xs : sg.ys, rcnt = rows_x ? sg.xcount : sg.ycount;
  const int64_t cbase = cols_x ? sg.xs : sg.ys, ccnt = cols_x ? sg.xcount : sg.ycount;
  const float *Gr = rows_x ? A.Gx : A.Gy;
  const float *Ar = rows_x ? A.Ax : A.Ay;
  const float *Gc = cols_x ? A.Gx : A.Gy;
  const float *Ac = cols_x ? A.Ax : A.Ay;
  float *acc = rows_x ? A.accX : A.accY;
  const bool crossb = (o == 0 || o == 3);
  const int toff = crossb ? DP : 0, soff = 2 * DP + (crossb ? 1 : 0);
  const bool self = (o == 1 || o == 2);

  const int tid = threadIdx.x;
  const int64_t row = (int64_t)item.tile * kGenRows + tid;
  const bool rv = row < rcnt;
  float xr[DP];
#pragma unroll
  for (int d = 0; d < DP; ++d) xr[d] = rv ? Gr[(rbase + row) * DP + d] : 0.f;
  const float a = rv ? Ar[rbase + row] : 0.f;
  float s = 0.f, sg2 = 0.f;
  float T[DP];
#pragma unroll
  for (int d = 0; d < DP; ++d) T[d] = 0.f;
  double s64 = 0.0, sg64 = 0.0;

  for (int64_t j0 = 0; j0 < ccnt; j0 += kGenCols) {
    __syncthreads();
    for (int e = tid; e < kGenCols * DP; e += kGenRows) {
      const int jj = e / DP, d = e % DP;
      const int64_t j = j0 + jj;
      ycol[e] = j < ccnt ? Gc[(cbase + j) * DP + d] : 0.f;
    }
    for (int jj = tid; jj < kGenCols; jj += kGenRows) {
      const int64_t j = j0 + jj;
      bcol[jj] = j < ccnt ? Ac[cbase + j] : 0.f;
    }
    __syncthreads();
    float st = 0.f, sgt = 0.f;
    // Only the column tiles that meet this CTA's rows in a self block hold
    // diagonal terms; they take the predicated loop, all others the plain one.
    const int64_t r0 = (int64_t)item.tile * kGenRows;
    if (self && j0 < r0 + kGenRows && j0 + kGenCols > r0) {
      const int64_t dj = row - j0;  // column of this row's diagonal term in the tile
      const int diag = (dj >= 0 && dj < kGenCols) ? (int)dj : -1;
      gen_cols<DP, MODE, true>(ycol, bcol, xr, T, st, sgt, diag);
    } else {
      gen_cols<DP, MODE, false>(ycol, bcol, xr, T, st, sgt, -1);
    }
    s += st;
    s64 += (double)st;
    if (SIG) sg64 += (double)sgt;
  }
  (void)sg2;
  if (MODE >= 1 && A.need_rows && rv) {
    float *dst = acc + (rbase + row) * gen_acc_stride(DP);
    dst[soff] = s;
#pragma unroll
    for (int d = 0; d < DP; ++d) dst[toff + d] = T[d];
  }
  // pair partials: K from x-y, x-x and y-y only (y-x would count Kxy twice);
  // a self block adds the diagonal a_i * a_i * k_ii = a_i^2 here
  double kv = (double)a * (s64 + (self ? (double)a : 0.0)), sv = (double)a * sg64;
  kv = warp_sum(kv);
  sv = warp_sum(sv);
  const int lane = tid & 31, wid = tid >> 5;
  if (lane == 0) {
    red[wid] = kv;
    red[kGenRows / 32 + wid] = sv;
  }
  __syncthreads();
  if (tid == 0) {
    double K = 0.0, S = 0.0;
    for (int w = 0; w < kGenRows / 32; ++w) {
      K += red[w];
      S += red[kGenRows / 32 + w];
    }
    A.itemK[it] = o == 3 ? 0.0 : K;
    A.itemS[it] = o == 3 ? 0.0 : S;
  }
}

}  // namespace ra
