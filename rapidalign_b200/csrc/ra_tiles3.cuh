// ra_tiles3.cuh -- the hot kernel for point clouds with D <= 3.
//
// Computes, for every pair and every block (x-y, x-x, y-y), the Gaussian
// kernel terms k = 2^(-|x' - y'|^2) on pre-scaled coordinates
// (x' = sqrt(log2(e) / (2 sigma^2)) * (x - anchor), so k = exp(-|x-y|^2/(2 sigma^2)),
// rapidalign/kde_gradients.py:32-36) and reduces them into
//   * per-item fp64 partials of K = sum a_i b_j k  (and of S = sum a b k r^2),
//   * per-point fp32 row sums for the backward:
//       s_i = sum_j b_j k_ij,   T_i = sum_j b_j y'_j k_ij     (rows)
//       s_j = sum_i a_i k_ij,   T_j = sum_i a_i x'_i k_ij     (columns)
//     from which the epilogue forms G_i = x'_i s_i - T_i = sum_j b_j k_ij (x'_i - y'_j).
// One pass over the UNIQUE terms: the self blocks visit only tiles J >= I;
// off-diagonal tiles feed both their rows and their columns, the diagonal
// tile is evaluated in full feeding only its rows.
//
// Work decomposition (B200: 148 SMs, FP32-pipe bound): a persistent grid of
// independent warps pulls items (pair, block, 64-row tile, column split) from
// a global ticket.  Inside a warp the 32 lanes form 4 rings of 8 lanes.  Every
// ring holds the same 64 rows (8 per lane, as 4 packed row pairs) and owns 16
// of the 64 columns of the current column tile; the column accumulators
// travel around the ring (one shuffle per step), so each column sum is
// complete after 8 steps without any cross-lane reduction arithmetic.  Row
// accumulators are combined across the 4 rings once per item.
//
// Data come from the padded tile layout written by pack3_kernel
// (ra_prep.cuh): a column is one 16-byte slot in each of the tile's NQ
// arrays, every slot of a padded tile exists and padding carries zero
// weight, so the inner loop has no bounds tests and addresses all loads of a
// step at immediate offsets from one pointer.
//
// Arithmetic per unique term (fwd+bwd): 3 sub + 3 mul/fma (r^2) + 1 EX2 +
// 4 FMA (row s, T) + 4 FMA (column s, T) = 14 FP32-pipe ops, issued as
// packed f32x2 instructions where both lanes of a row pair share operands.
// Row sums accumulate in fp32 over an item (at most 4096 columns) and are
// folded once into the fp64 K and S partials, which are reduced in a fixed
// order; only the per-point fp32 red.add at L2 depends on timing.  The next
// column tile is prefetched into L1 while the current one is processed.
#pragma once

#include "ra_common.cuh"


namespace ra {

// 4 warps per CTA, 3 CTAs (12 warps) per SM at <= 168 registers: measured
// best on B200 against 14-16 warps at 128 registers (which spill).
constexpr int kT3Threads = 128;
#ifndef RA_T3_MINB
#define RA_T3_MINB 3
#endif
constexpr int kT3MinBlocks = RA_T3_MINB;

struct Tiles3Args {
  const Item *items;
  const int64_t *n_items;  // device scalar
  unsigned int *ticket;    // zeroed before the launch
  const Seg *seg;
  const int64_t *tbase_x, *tbase_y;     // first tile of each pair's cloud
  const ulonglong2 *tiles_x, *tiles_y;  // [tiles][NQ][64]
  float *acc_x, *acc_y;                 // [tiles * 64][8]: self (s, T0..T2), cross (s, T0..T2)
  double *itemK, *itemS;
  int shard_index, shard_count;  // this process evaluates items shard_index + k * shard_count
};

// MODE 0: K only.  MODE 1: K + per-point sums.  MODE 2: also S (sigma grad).
template <int MODE>
struct Tiles3Mode {
  static constexpr bool GRAD = MODE >= 1;
  static constexpr bool SIG = MODE == 2;
  static constexpr int NQ = GRAD ? 4 : 2;
};

template <int MODE, bool DIAG>
__device__ __forceinline__ void tiles3_coltile(
    const ulonglong2 *__restrict__ ct, const int col0, const int ccnt,
    float *__restrict__ accC, const int lane, const f2_t (&X0)[4], const f2_t (&X1)[4],
    const f2_t (&X2)[4], const f2_t (&Aw)[4], const f2_t (&AX0)[4], const f2_t (&AX1)[4],
    const f2_t (&AX2)[4], f2_t (&st)[4], f2_t (&T0)[4], f2_t (&T1)[4], f2_t (&T2)[4],
    f2_t (&sgt)[4]) {
  constexpr bool GRAD = Tiles3Mode<MODE>::GRAD;
  constexpr bool SIG = Tiles3Mode<MODE>::SIG;
  constexpr bool COLS = GRAD && !DIAG;
  const int q = lane >> 3, p = lane & 7;
  const int ring_base = lane & ~7;
  float cs[2], c0[2], c1[2], c2[2];
#pragma unroll
  for (int c = 0; c < 2; ++c) cs[c] = c0[c] = c1[c] = c2[c] = 0.f;

#pragma unroll 1
  for (int t = 0; t < 8; ++t) {
    const ulonglong2 *cp = ct + q * 8 + ((p + t) & 7);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const ulonglong2 q0 = cp[c * 32];
      const ulonglong2 q1 = cp[c * 32 + kTile];
      ulonglong2 q2 = make_ulonglong2(0ull, 0ull), q3 = q2;
      if (GRAD) {
        q2 = cp[c * 32 + 2 * kTile];
        q3 = cp[c * 32 + 3 * kTile];
      }
      const f2_t Y0 = q0.x, Y1 = q0.y, Y2 = q1.x, B = q1.y;
#pragma unroll
      for (int rp = 0; rp < 4; ++rp) {
        const f2_t dx = sub2(X0[rp], Y0);
        const f2_t dy = sub2(X1[rp], Y1);
        const f2_t dz = sub2(X2[rp], Y2);
        f2_t r2 = mul2(dx, dx);
        r2 = fma2(dy, dy, r2);
        r2 = fma2(dz, dz, r2);
        float r_lo, r_hi;
        upk(r2, r_lo, r_hi);
        const float k_lo = ex2(-r_lo), k_hi = ex2(-r_hi);
        const f2_t k = pk(k_lo, k_hi);
        if (SIG) {
          const f2_t wk = mul2(B, k);
          st[rp] = add2(st[rp], wk);
          sgt[rp] = fma2(wk, r2, sgt[rp]);
        } else {
          st[rp] = fma2(B, k, st[rp]);
        }
        if (GRAD) {
          T0[rp] = fma2(q2.x, k, T0[rp]);
          T1[rp] = fma2(q2.y, k, T1[rp]);
          T2[rp] = fma2(q3.x, k, T2[rp]);
        }
        if (COLS) {
          float a_lo, a_hi;
          upk(Aw[rp], a_lo, a_hi);
          cs[c] = fmaf(a_lo, k_lo, cs[c]);
          cs[c] = fmaf(a_hi, k_hi, cs[c]);
          upk(AX0[rp], a_lo, a_hi);
          c0[c] = fmaf(a_lo, k_lo, c0[c]);
          c0[c] = fmaf(a_hi, k_hi, c0[c]);
          upk(AX1[rp], a_lo, a_hi);
          c1[c] = fmaf(a_lo, k_lo, c1[c]);
          c1[c] = fmaf(a_hi, k_hi, c1[c]);
          upk(AX2[rp], a_lo, a_hi);
          c2[c] = fmaf(a_lo, k_lo, c2[c]);
          c2[c] = fmaf(a_hi, k_hi, c2[c]);
        }
      }
    }
    if (COLS && t < 7) {
      // pass the column accumulators one position back around the ring
      const int src = ring_base | ((p + 1) & 7);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        cs[c] = __shfl_sync(kFull, cs[c], src);
        c0[c] = __shfl_sync(kFull, c0[c], src);
        c1[c] = __shfl_sync(kFull, c1[c], src);
        c2[c] = __shfl_sync(kFull, c2[c], src);
      }
    }
  }
  if (COLS) {
    // after step 7 this lane holds the sums of position (p + 7) & 7
    const int pos = (p + 7) & 7;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int in_tile = c * 32 + q * 8 + pos;
      if (col0 + in_tile < ccnt) red_add_v4(accC + in_tile * kAcc3Stride, cs[c], c0[c], c1[c], c2[c]);
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(kT3Threads, kT3MinBlocks) tiles3_kernel(Tiles3Args A) {
  constexpr bool GRAD = Tiles3Mode<MODE>::GRAD;
  constexpr bool SIG = Tiles3Mode<MODE>::SIG;
  constexpr int NQ = Tiles3Mode<MODE>::NQ;
  constexpr int TILE_U2 = NQ * kTile;  // 16-byte slots per tile
  const int lane = threadIdx.x & 31;
  const int q = lane >> 3, p = lane & 7;
  const int64_t total = *A.n_items;
  for (;;) {
    unsigned ticket = 0;
    if (lane == 0) ticket = atomicAdd(A.ticket, 1u);
    ticket = __shfl_sync(kFull, ticket, 0);
    const int64_t it = A.shard_index + (int64_t)ticket * A.shard_count;
    if (it >= total) break;
    const Item item = A.items[it];
    const Seg sg = A.seg[item.pair];
    const int blk = item.block;
    const bool sym = blk != 0;
    const bool rows_y = blk == 2, cols_x = blk == 1;
    const int64_t rcnt = rows_y ? sg.ycount : sg.xcount;
    const int64_t ccnt = cols_x ? sg.xcount : sg.ycount;
    const int64_t rtb = (rows_y ? A.tbase_y : A.tbase_x)[item.pair];
    const int64_t ctb = (cols_x ? A.tbase_x : A.tbase_y)[item.pair];
    const ulonglong2 *__restrict__ rt = rows_y ? A.tiles_y : A.tiles_x;
    const ulonglong2 *__restrict__ ctiles = cols_x ? A.tiles_x : A.tiles_y;
    float *accR = rows_y ? A.acc_y : A.acc_x;
    float *accC = cols_x ? A.acc_x : A.acc_y;
    const int off = blk == 0 ? kAcc3Block : 0;  // cross block after the self block

    // 32-bit tile/column indices: a pair's cloud has < 2^31 points
    const int nTc = (int)ceil_div(ccnt, (int64_t)kTile);
    const int S = (int)splits_for(nTc);
    const int L = (nTc + S - 1) / S;
    const int I = item.tile;
    int J0 = item.split * L;
    const int J1 = J0 + L < nTc ? J0 + L : nTc;
    if (sym && J0 < I) J0 = I;
    if (J0 >= J1) {
      if (lane == 0) {
        A.itemK[it] = 0.0;
        A.itemS[it] = 0.0;
      }
      continue;
    }
    const int cc = (int)ccnt;
    const ulonglong2 *__restrict__ ct0 = ctiles + ctb * TILE_U2;  // the pair's first column tile
    float *accC0 = accC + ctb * (kTile * kAcc3Stride) + off;

    // ---- rows: 8 per lane as 4 packed pairs (padding rows have zero weight) --
    f2_t X0[4], X1[4], X2[4], Aw[4], AX0[4], AX1[4], AX2[4];
    {
      const ulonglong2 *rp0 = rt + (rtb + I) * TILE_U2 + p * 8;
#pragma unroll
      for (int rp = 0; rp < 4; ++rp) {
        const ulonglong2 a0 = rp0[2 * rp], b0 = rp0[2 * rp + 1];                  // x', y'
        const ulonglong2 a1 = rp0[kTile + 2 * rp], b1 = rp0[kTile + 2 * rp + 1];  // z', a
        X0[rp] = pk(lo_of(a0.x), lo_of(b0.x));
        X1[rp] = pk(lo_of(a0.y), lo_of(b0.y));
        X2[rp] = pk(lo_of(a1.x), lo_of(b1.x));
        Aw[rp] = pk(lo_of(a1.y), lo_of(b1.y));
        if (GRAD) {
          const ulonglong2 a2 = rp0[2 * kTile + 2 * rp], b2 = rp0[2 * kTile + 2 * rp + 1];
          const ulonglong2 a3 = rp0[3 * kTile + 2 * rp], b3 = rp0[3 * kTile + 2 * rp + 1];
          AX0[rp] = pk(lo_of(a2.x), lo_of(b2.x));
          AX1[rp] = pk(lo_of(a2.y), lo_of(b2.y));
          AX2[rp] = pk(lo_of(a3.x), lo_of(b3.x));
        } else {
          AX0[rp] = AX1[rp] = AX2[rp] = 0ull;
        }
      }
    }
    f2_t st[4], T0[4], T1[4], T2[4], sgt[4];
    const f2_t z2 = pk(0.f, 0.f);
#pragma unroll
    for (int rp = 0; rp < 4; ++rp) st[rp] = T0[rp] = T1[rp] = T2[rp] = sgt[rp] = z2;
    double ktot = 0.0, kd = 0.0, stot_sig = 0.0, sd = 0.0;

    // ---- the diagonal tile of a self block first (rows only, counted once) --
    if (sym && J0 == I) {
      tiles3_coltile<MODE, true>(ct0 + I * TILE_U2, I * kTile, cc,
                                 accC0 + I * (kTile * kAcc3Stride), lane, X0, X1, X2, Aw, AX0,
                                 AX1, AX2, st, T0, T1, T2, sgt);
#pragma unroll
      for (int rp = 0; rp < 4; ++rp) {
        float s_lo, s_hi, a_lo, a_hi;
        upk(st[rp], s_lo, s_hi);
        upk(Aw[rp], a_lo, a_hi);
        kd = fma((double)a_lo, (double)s_lo, kd);
        kd = fma((double)a_hi, (double)s_hi, kd);
        if (SIG) {
          upk(sgt[rp], s_lo, s_hi);
          sd = fma((double)a_lo, (double)s_lo, sd);
          sd = fma((double)a_hi, (double)s_hi, sd);
        }
      }
      ++J0;
    }
    // ---- off-diagonal tiles: rows and columns ------------------------------
#pragma unroll 1
    for (int J = J0; J < J1; ++J) {
      const ulonglong2 *ct = ct0 + J * TILE_U2;
      if (J + 1 < J1) {
        // one 128-byte line per lane covers the next tile (NQ * 64 * 16 bytes)
        const char *nxt = reinterpret_cast<const char *>(ct + TILE_U2);
        for (int l = lane; l < TILE_U2 / 8; l += 32)
          asm volatile("prefetch.global.L1 [%0];" ::"l"(nxt + l * 128));
      }
      tiles3_coltile<MODE, false>(ct, J * kTile, cc, accC0 + J * (kTile * kAcc3Stride), lane,
                                  X0, X1, X2, Aw, AX0, AX1, AX2, st, T0, T1, T2, sgt);
    }
    // row sums accumulated in fp32 over the item: fold once into fp64
#pragma unroll
    for (int rp = 0; rp < 4; ++rp) {
      float s_lo, s_hi, a_lo, a_hi;
      upk(st[rp], s_lo, s_hi);
      upk(Aw[rp], a_lo, a_hi);
      ktot = fma((double)a_lo, (double)s_lo, ktot);
      ktot = fma((double)a_hi, (double)s_hi, ktot);
      if (SIG) {
        upk(sgt[rp], s_lo, s_hi);
        stot_sig = fma((double)a_lo, (double)s_lo, stot_sig);
        stot_sig = fma((double)a_hi, (double)s_hi, stot_sig);
      }
    }

    // ---- pair partials: off-diagonal self terms count twice ----------------
    const double kl = sym ? 2.0 * ktot - kd : ktot;
    const double kw = warp_sum(kl);
    double sw = 0.0;
    if (SIG) sw = warp_sum(sym ? 2.0 * stot_sig - sd : stot_sig);
    if (lane == 0) {
      A.itemK[it] = kw;
      A.itemS[it] = sw;
    }

    // ---- per-point row sums: combine the 4 rings, then one lane per row ----
    if (GRAD) {
#pragma unroll
      for (int rp = 0; rp < 4; ++rp) {
#pragma unroll
        for (int o = 8; o <= 16; o <<= 1) {
          st[rp] = add2(st[rp], __shfl_xor_sync(kFull, st[rp], o));
          T0[rp] = add2(T0[rp], __shfl_xor_sync(kFull, T0[rp], o));
          T1[rp] = add2(T1[rp], __shfl_xor_sync(kFull, T1[rp], o));
          T2[rp] = add2(T2[rp], __shfl_xor_sync(kFull, T2[rp], o));
        }
      }
      float *accI = accR + ((rtb + I) * kTile) * kAcc3Stride + off;
#pragma unroll
      for (int rp = 0; rp < 4; ++rp) {
        if (rp == q) {
          const int r0 = p * 8 + 2 * rp;
          float s_lo, s_hi, t0l, t0h, t1l, t1h, t2l, t2h;
          upk(st[rp], s_lo, s_hi);
          upk(T0[rp], t0l, t0h);
          upk(T1[rp], t1l, t1h);
          upk(T2[rp], t2l, t2h);
          if ((int64_t)I * kTile + r0 < rcnt) red_add_v4(accI + r0 * kAcc3Stride, s_lo, t0l, t1l, t2l);
          if ((int64_t)I * kTile + r0 + 1 < rcnt)
            red_add_v4(accI + (r0 + 1) * kAcc3Stride, s_hi, t0h, t1h, t2h);
        }
      }
    }
  }
}

}  // namespace ra
