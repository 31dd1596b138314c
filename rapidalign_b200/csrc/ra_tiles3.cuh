// ra_tiles3.cuh -- the hot kernel for point clouds with D <= 3.
//
// Computes, for every pair and every block (x-y, x-x, y-y), the Gaussian
// kernel terms k = 2^(-|x' - y'|^2) on pre-scaled coordinates
// (x' = sqrt(log2(e) / (2 sigma^2)) * (x - anchor), so k = exp(-|x-y|^2/(2 sigma^2)),
// rapidalign/kde_gradients.py:32-36) and reduces them into
//   * per-item fp64 partials of K = sum a_i b_j k  (and of S = sum a b k r^2),
//   * per-point fp32 sums for the backward, in difference form:
//       s_i = sum_j b_j k_ij,   G_i = sum_j b_j k_ij (x'_i - y'_j)      (rows)
//       s_j = sum_i a_i k_ij,   G_j = sum_i a_i k_ij (y'_j - x'_i)      (columns)
//     (kde_gradients.py:98-113 needs exactly these: dK/dx_i = -(w_i/sigma^2) G_i).
// The differences x' - y' are the ones already formed for r^2, so the sums
// carry no cancellation however far the clouds sit from the origin.
// One pass over the UNIQUE terms: the self blocks visit only tiles J >= I;
// off-diagonal tiles feed both their rows and their columns, the diagonal
// tile is evaluated in full feeding only its rows.
//
// Work decomposition (B200: 148 SMs, FP32-pipe bound): a persistent grid of
// independent warps pulls items (pair, block, 64-row tile, column split) from
// a global ticket, in the plan's order (ra_plan.cuh: the largest pairs first,
// each pair's items together, so neighbouring items share column tiles in
// L2).  Inside a warp the 32 lanes form 4 rings of 8 lanes.  Every
// ring holds the same 64 rows (8 per lane, as 4 packed row pairs) and owns 16
// of the 64 columns of the current column tile; the column accumulators
// travel around the ring (one shuffle per step), so each column sum is
// complete after 8 steps without any cross-lane reduction arithmetic.  Row
// accumulators are combined across the 4 rings once per item.
//
// Data come from the padded tile layout written by pack3_kernel
// (ra_prep.cuh): a column is one 16-byte slot in each of the tile's two
// arrays ({x',x',y',y'}, {z',z',w,w}), every slot of a padded tile exists and
// padding carries zero weight, so the inner loop has no bounds tests and
// addresses the loads of a step at immediate offsets from one pointer.  The
// next column tile is prefetched into L1 while the current one is processed.
//
// Arithmetic per unique term (fwd+bwd): 3 sub + 3 mul/fma (r^2) + 1 EX2 +
// w = b k, s += w, G += w d (5) for the row + the same 5 for the column =
// 16 FP32-pipe operations, issued mostly as packed f32x2 instructions in
// which the two rows of a row pair share the column operand.  When the
// column cloud's weights are all >= 0 they are folded into the exponent:
// the column slot holds -log2(b~_j) (b~ = b / max b), the r^2 chain starts
// from it instead of a plain product, and EX2 returns w = b~_j k directly,
// which drops the row-side multiply: 15 operations per unique term.  The
// per-point sums then carry the factor 1 / max b of the partner cloud,
// which the epilogue restores.  When the row cloud's weights are moreover all
// equal (a~ = 1, padding rows far away so that their k is 0) the column-side
// multiply by a~_i goes too: 14 operations per unique term.
// Row sums accumulate in fp32 over an item (at most 4096 columns) and are
// folded once into the fp64 K and S partials, which are reduced in a fixed
// order; only the per-point fp32 red.add at L2 depends on timing.
#pragma once

#include "ra_common.cuh"
#include "ra_prep.cuh"

namespace ra {

// Column tiles are staged in shared memory by cp.async, NSTAGE buffers per
// warp (the next tiles in flight while one is used; 3 measured 0.6 % faster
// than 2); RA_T3_SMEM=0 builds the variant that reads them through L1 after
// a prefetch instead (measured 4.7 % slower on the 4096-graph batch).
#ifndef RA_T3_SMEM
#define RA_T3_SMEM 1
#endif
#ifndef RA_T3_NSTAGE
#define RA_T3_NSTAGE 3
#endif
#if RA_T3_SMEM
constexpr int kT3Stages = RA_T3_NSTAGE;
__shared__ __align__(16) ulonglong2 t3_stage[4][kT3Stages][2 * kTile];  // 4 warps per CTA
// the warp copies one column tile (128 chunks of 16 bytes) into `dst`
__device__ __forceinline__ void t3_stage_tile(ulonglong2 *dst, const ulonglong2 *src, int lane) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int c = lane + 32 * k;
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst + c);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src + c) : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}
#endif

template <bool V>
struct BoolTag {
  static constexpr bool value = V;
};

// 4 warps per CTA, 3 CTAs (12 warps) per SM at <= 168 registers.
constexpr int kT3Threads = 128;
#ifndef RA_T3_MINB
#define RA_T3_MINB 3
#endif
constexpr int kT3MinBlocks = RA_T3_MINB;
constexpr int kT3Arrays = 2;  // 16-byte arrays per tile: {x',x',y',y'}, {z',z',w,w}
constexpr int kT3TileU2 = kT3Arrays * kTile;

struct Tiles3Args {
  const Item *items;
  const int64_t *n_items;  // device scalar
  unsigned int *ticket;    // zeroed before the launch
  const Seg *seg;
  const int64_t *tbase_x, *tbase_y;     // first tile of each pair's cloud
  const ulonglong2 *tiles_x, *tiles_y;  // [tiles][2][64]
  const float *aw_x, *aw_y;             // [tiles * 64] a~ = a / m per slot
  const double *meta;                   // per-pair metadata (ra_prep.cuh)
  float *acc_x, *acc_y;                 // [tiles * 64][8]: self (s, G0..G2), cross (s, G0..G2)
  double *itemK, *itemS;
  int shard_index, shard_count;  // this process evaluates items shard_index + k * shard_count
  const int32_t *order;          // ticket k takes item order[k] (null: item k)
};

// MODE 0: K only.  MODE 1: K + per-point sums.  MODE 2: also S (sigma grad).
// MODE 3: as MODE 1 without the columns' weight sums s_j, which only the
// weight gradients need (one FP32 operation and one shuffle fewer per term).
template <int MODE>
struct Tiles3Mode {
  static constexpr bool GRAD = MODE >= 1;
  static constexpr bool SIG = MODE == 2;
  static constexpr bool CSUM = MODE == 1 || MODE == 2;  // column weight sums
};

// One column half (32 columns: 8 per ring position) against the lane's 4 row
// pairs: updates the row sums and this half's travelling column sums.
// FOLD: the column's fourth value is -log2(b~) (see the file comment).
// RUNI: every row has a~ = 1 (or is padding with k = 0).
template <int MODE, bool COLS, bool FOLD, bool RUNI = false>
__device__ __forceinline__ void t3_half(const ulonglong2 q0, const ulonglong2 q1,
                                        const f2_t (&X0)[4], const f2_t (&X1)[4],
                                        const f2_t (&X2)[4], const f2_t (&Aw)[4], f2_t (&st)[4],
                                        f2_t (&G0)[4], f2_t (&G1)[4], f2_t (&G2)[4],
                                        f2_t (&sgt)[4], f2_t &cs, f2_t &c0, f2_t &c1, f2_t &c2) {
  constexpr bool GRAD = Tiles3Mode<MODE>::GRAD;
  constexpr bool SIG = Tiles3Mode<MODE>::SIG;
  const f2_t Y0 = q0.x, Y1 = q0.y, Y2 = q1.x, B = q1.y;
#pragma unroll
  for (int rp = 0; rp < 4; ++rp) {
    const f2_t dx = sub2(X0[rp], Y0);
    const f2_t dy = sub2(X1[rp], Y1);
    const f2_t dz = sub2(X2[rp], Y2);
    f2_t r2 = FOLD ? fma2(dx, dx, B) : mul2(dx, dx);
    r2 = fma2(dy, dy, r2);
    r2 = fma2(dz, dz, r2);
    float r_lo, r_hi;
    upk(r2, r_lo, r_hi);
    const f2_t k = pk(ex2(-r_lo), ex2(-r_hi));  // FOLD: b~_j k_ij
    if (GRAD) {
      const f2_t w = FOLD ? k : mul2(B, k);  // b_j k_ij for the two rows
      st[rp] = add2(st[rp], w);
      G0[rp] = fma2(w, dx, G0[rp]);
      G1[rp] = fma2(w, dy, G1[rp]);
      G2[rp] = fma2(w, dz, G2[rp]);
      if (SIG) sgt[rp] = fma2(w, r2, sgt[rp]);  // never folded: r2 is r^2
    } else {
      st[rp] = FOLD ? add2(st[rp], k) : fma2(B, k, st[rp]);
    }
    if (COLS) {
      const f2_t wc = RUNI ? k : mul2(Aw[rp], k);  // a_i k_ij for the two rows
      if (Tiles3Mode<MODE>::CSUM) cs = add2(cs, wc);
      c0 = fma2(wc, dx, c0);
      c1 = fma2(wc, dy, c1);
      c2 = fma2(wc, dz, c2);
    }
  }
}

// Pass a half's column sums one position back around the ring.
template <bool CSUM>
__device__ __forceinline__ void t3_rotate(f2_t &cs, f2_t &c0, f2_t &c1, f2_t &c2, int src) {
  if (CSUM) cs = __shfl_sync(kFull, cs, src);
  c0 = __shfl_sync(kFull, c0, src);
  c1 = __shfl_sync(kFull, c1, src);
  c2 = __shfl_sync(kFull, c2, src);
}

// One 64-column tile against the warp's 64 rows.  The 8 ring steps are fully
// unrolled and each half's column sums are rotated as soon as that half is
// done, so the shuffles of one half overlap the arithmetic of the other and
// the steps interleave (6 % faster than a rolled loop that rotates both
// halves at the end of a step).
template <int MODE, bool DIAG, bool FOLD, bool RUNI = false>
__device__ __forceinline__ void tiles3_coltile(
    const ulonglong2 *__restrict__ ct, const int col0, const int ccnt,
    float *__restrict__ accC, const int lane, const f2_t (&X0)[4], const f2_t (&X1)[4],
    const f2_t (&X2)[4], const f2_t (&Aw)[4], f2_t (&st)[4], f2_t (&G0)[4], f2_t (&G1)[4],
    f2_t (&G2)[4], f2_t (&sgt)[4]) {
  constexpr bool GRAD = Tiles3Mode<MODE>::GRAD;
  constexpr bool COLS = GRAD && !DIAG;
  const int q = lane >> 3, p = lane & 7;
  const int src = (lane & ~7) | ((p + 1) & 7);
  f2_t cs[2], c0[2], c1[2], c2[2];  // {sum over even rows, sum over odd rows}
#pragma unroll
  for (int c = 0; c < 2; ++c) cs[c] = c0[c] = c1[c] = c2[c] = 0ull;
  const ulonglong2 *cb = ct + q * 8;
  if (!COLS) {
    // rows only (forward-only runs and the diagonal tile): nothing travels,
    // and the rolled loop is the faster one here (3.35 vs 3.73 ms, K-only)
#pragma unroll 1
    for (int t = 0; t < 8; ++t) {
      const ulonglong2 *cp = cb + ((p + t) & 7);
      const ulonglong2 a00 = cp[0], a01 = cp[kTile], a10 = cp[32], a11 = cp[32 + kTile];
      t3_half<MODE, false, FOLD>(a00, a01, X0, X1, X2, Aw, st, G0, G1, G2, sgt, cs[0], c0[0],
                                 c1[0], c2[0]);
      t3_half<MODE, false, FOLD>(a10, a11, X0, X1, X2, Aw, st, G0, G1, G2, sgt, cs[1], c0[1],
                                 c1[1], c2[1]);
    }
    return;
  }
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const ulonglong2 *cp = cb + ((p + t) & 7);
    const ulonglong2 a00 = cp[0], a01 = cp[kTile], a10 = cp[32], a11 = cp[32 + kTile];
    t3_half<MODE, COLS, FOLD, RUNI>(a00, a01, X0, X1, X2, Aw, st, G0, G1, G2, sgt, cs[0], c0[0],
                                    c1[0], c2[0]);
    if (t < 7) t3_rotate<Tiles3Mode<MODE>::CSUM>(cs[0], c0[0], c1[0], c2[0], src);
    t3_half<MODE, COLS, FOLD, RUNI>(a10, a11, X0, X1, X2, Aw, st, G0, G1, G2, sgt, cs[1], c0[1],
                                    c1[1], c2[1]);
    if (t < 7) t3_rotate<Tiles3Mode<MODE>::CSUM>(cs[1], c0[1], c1[1], c2[1], src);
  }
  {
    // after step 7 this lane holds the sums of position (p + 7) & 7; the
    // columns' own differences are y'_j - x'_i, hence the sign.  Folded
    // columns carry b~_j in every term: divide it out (2^(-log2 b~_j)).
    const int pos = (p + 7) & 7;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int in_tile = c * 32 + q * 8 + pos;
      float vs = lo_of(cs[c]) + hi_of(cs[c]), v0 = lo_of(c0[c]) + hi_of(c0[c]);
      float v1 = lo_of(c1[c]) + hi_of(c1[c]), v2 = lo_of(c2[c]) + hi_of(c2[c]);
      if (col0 + in_tile < ccnt) {
        if (FOLD) {
          const float inv = ex2(lo_of(ct[kTile + in_tile].y));
          vs *= inv;
          v0 *= inv;
          v1 *= inv;
          v2 *= inv;
        }
        red_add_v4(accC + in_tile * kAcc3Stride, vs, -v0, -v1, -v2);
      }
    }
  }
}

// ROWS (the deterministic mode): every block is evaluated in both
// orientations with row sums only -- items of blocks 0 (x rows, y columns),
// 1 (x, x), 2 (y, y) and 3 (y rows, x columns), all column tiles, no column
// splits -- so each point's record is written by exactly one item with plain
// stores: no atomic addition anywhere, results independent of scheduling.
// Costs about 1.5x the FP32 work of the symmetric default (10 operations per
// term, every term twice, against 13-15 per unique term).
template <int MODE, bool ROWS = false>
__global__ void __launch_bounds__(kT3Threads, kT3MinBlocks) tiles3_kernel(Tiles3Args A) {
  constexpr bool GRAD = Tiles3Mode<MODE>::GRAD;
  constexpr bool SIG = Tiles3Mode<MODE>::SIG;
  const int lane = threadIdx.x & 31;
  const int q = lane >> 3, p = lane & 7;
  const int64_t total = *A.n_items;
  for (;;) {
    unsigned ticket = 0;
    if (lane == 0) ticket = atomicAdd(A.ticket, 1u);
    ticket = __shfl_sync(kFull, ticket, 0);
    const int64_t k = A.shard_index + (int64_t)ticket * A.shard_count;
    if (k >= total) break;
    const int64_t it = A.order != nullptr ? A.order[k] : k;  // largest pairs first
    if (it < 0 || it >= total) continue;  // (an order entry the plan could not write)
    const Item item = A.items[it];
    const Seg sg = A.seg[item.pair];
    const int blk = item.block;
    const bool sym = !ROWS && blk != 0;  // a self block visited as its upper triangle
    const bool rows_y = blk == 2 || blk == 3, cols_x = blk == 1 || blk == 3;
    const int64_t rcnt = rows_y ? sg.ycount : sg.xcount;
    const int64_t ccnt = cols_x ? sg.xcount : sg.ycount;
    const int64_t rtb = (rows_y ? A.tbase_y : A.tbase_x)[item.pair];
    const int64_t ctb = (cols_x ? A.tbase_x : A.tbase_y)[item.pair];
    const ulonglong2 *__restrict__ rt = rows_y ? A.tiles_y : A.tiles_x;
    const ulonglong2 *__restrict__ ctiles = cols_x ? A.tiles_x : A.tiles_y;
    float *accR = rows_y ? A.acc_y : A.acc_x;
    float *accC = cols_x ? A.acc_x : A.acc_y;
    const int off = (blk == 0 || blk == 3) ? kAcc3Block : 0;  // cross block after the self
    const float *__restrict__ awr = rows_y ? A.aw_y : A.aw_x;
    const double *meta = A.meta + item.pair * (int64_t)meta_stride(3);
    const int rside = rows_y ? 1 : 0, cside = cols_x ? 0 : 1;
    // the column weights are folded into the exponent when all >= 0 (never
    // with the sigma gradient, whose r^2 the fold would shift)
    const bool fold = !SIG && meta[meta_fold(3) + cside] != 0.0;
    const bool runi = fold && meta[meta_fold(3) + rside] == 2.0;

    // 32-bit tile/column indices: a pair's cloud has < 2^31 points
    const int nTc = (int)ceil_div(ccnt, (int64_t)kTile);
    const int S = ROWS ? 1 : (int)splits_for(nTc);
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
    const ulonglong2 *__restrict__ ct0 = ctiles + ctb * kT3TileU2;  // the pair's first column tile
    float *accC0 = accC + ctb * (kTile * kAcc3Stride) + off;

    // ---- rows: 8 per lane as 4 packed pairs (padding rows have zero weight) --
    f2_t X0[4], X1[4], X2[4], Aw[4];
    const float4 *awp = reinterpret_cast<const float4 *>(awr + (rtb + I) * kTile + p * 8);
    // the rows' weights a~ (loaded again after the column loop, so that a
    // loop that does not use them -- equal weights -- holds no registers for them)
    auto load_aw = [&]() {
      const float4 aw0 = awp[0], aw1 = awp[1];
      const float awv[8] = {aw0.x, aw0.y, aw0.z, aw0.w, aw1.x, aw1.y, aw1.z, aw1.w};
#pragma unroll
      for (int rp = 0; rp < 4; ++rp) Aw[rp] = pk(awv[2 * rp], awv[2 * rp + 1]);
    };
    {
      const ulonglong2 *rp0 = rt + (rtb + I) * kT3TileU2 + p * 8;
#pragma unroll
      for (int rp = 0; rp < 4; ++rp) {
        const ulonglong2 a0 = rp0[2 * rp], b0 = rp0[2 * rp + 1];                  // x', y'
        const ulonglong2 a1 = rp0[kTile + 2 * rp], b1 = rp0[kTile + 2 * rp + 1];  // z', v
        X0[rp] = pk(lo_of(a0.x), lo_of(b0.x));
        X1[rp] = pk(lo_of(a0.y), lo_of(b0.y));
        X2[rp] = pk(lo_of(a1.x), lo_of(b1.x));
      }
      load_aw();
    }
    f2_t st[4], G0[4], G1[4], G2[4], sgt[4];
    const f2_t z2 = pk(0.f, 0.f);
#pragma unroll
    for (int rp = 0; rp < 4; ++rp) st[rp] = G0[rp] = G1[rp] = G2[rp] = sgt[rp] = z2;
    double ktot = 0.0, kd = 0.0, stot_sig = 0.0, sd = 0.0;

    // ---- the diagonal tile of a self block first (rows only, counted once) --
    if (sym && J0 == I) {
      if (fold)
        tiles3_coltile<MODE, true, !SIG>(ct0 + I * kT3TileU2, I * kTile, cc,
                                         accC0 + I * (kTile * kAcc3Stride), lane, X0, X1, X2, Aw,
                                         st, G0, G1, G2, sgt);
      else
        tiles3_coltile<MODE, true, false>(ct0 + I * kT3TileU2, I * kTile, cc,
                                          accC0 + I * (kTile * kAcc3Stride), lane, X0, X1, X2,
                                          Aw, st, G0, G1, G2, sgt);
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
    auto offdiag = [&](auto fold_tag, auto uni_tag) {
      constexpr bool F = decltype(fold_tag)::value;
      constexpr bool U = decltype(uni_tag)::value;
#if RA_T3_SMEM
      // the first kT3Stages - 1 tiles in flight; each step then starts the
      // copy of tile J + kT3Stages - 1 and waits for tile J (an empty copy
      // group keeps the count uniform near the end of the range)
      ulonglong2(*buf)[kT3TileU2] = t3_stage[threadIdx.x >> 5];
#pragma unroll
      for (int q = 0; q < kT3Stages - 1; ++q) {
        if (J0 + q < J1) t3_stage_tile(buf[q], ct0 + (J0 + q) * kT3TileU2, lane);
        else asm volatile("cp.async.commit_group;" ::: "memory");
      }
#endif
#pragma unroll 1
      for (int J = J0; J < J1; ++J) {
#if RA_T3_SMEM
        {
          const int Jn = J + kT3Stages - 1;
          if (Jn < J1) t3_stage_tile(buf[(Jn - J0) % kT3Stages], ct0 + Jn * kT3TileU2, lane);
          else asm volatile("cp.async.commit_group;" ::: "memory");
          asm volatile("cp.async.wait_group %0;" ::"n"(kT3Stages - 1) : "memory");
        }
        __syncwarp();
        const ulonglong2 *ct = buf[(J - J0) % kT3Stages];
#else
        const ulonglong2 *ct = ct0 + J * kT3TileU2;
        if (J + 1 < J1) {
          // 2 KB tile = 16 lines of 128 bytes: lanes 0..15 prefetch one each
          const char *nxt = reinterpret_cast<const char *>(ct + kT3TileU2);
          if (lane < kT3TileU2 / 8)
            asm volatile("prefetch.global.L1 [%0];" ::"l"(nxt + lane * 128));
        }
#endif
        // row sums: a fresh fp32 subtotal per tile, added to the item's
        // total (64-term then tile-count-long fp32 sums instead of one long one)
        f2_t stt[4];
#pragma unroll
        for (int rp = 0; rp < 4; ++rp) stt[rp] = z2;
        tiles3_coltile<MODE, ROWS, F, U>(ct, J * kTile, cc,
                                          accC0 + J * (kTile * kAcc3Stride), lane, X0, X1, X2,
                                          Aw, stt, G0, G1, G2, sgt);
#pragma unroll
        for (int rp = 0; rp < 4; ++rp) st[rp] = add2(st[rp], stt[rp]);
#if RA_T3_SMEM
        __syncwarp();  // every lane is done with this buffer before it is refilled
#endif
      }
    };
    if (runi)
      offdiag(BoolTag<!SIG>{}, BoolTag<!SIG>{});
    else if (fold)
      offdiag(BoolTag<!SIG>{}, BoolTag<false>{});
    else
      offdiag(BoolTag<false>{}, BoolTag<false>{});
    load_aw();  // a fresh load: the loop's atomics are memory barriers to the compiler
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
    // K = m_r m_c sum a~_i s~_i
    const double kscale = meta[meta_wscale(3) + rside] * meta[meta_wscale(3) + cside];
    if (lane == 0) {
      A.itemK[it] = kw * kscale;
      A.itemS[it] = sw * kscale;
    }

    // ---- per-point row sums: combine the 4 rings, then one lane per row ----
    if (GRAD) {
#pragma unroll
      for (int rp = 0; rp < 4; ++rp) {
#pragma unroll
        for (int o = 8; o <= 16; o <<= 1) {
          st[rp] = add2(st[rp], __shfl_xor_sync(kFull, st[rp], o));
          G0[rp] = add2(G0[rp], __shfl_xor_sync(kFull, G0[rp], o));
          G1[rp] = add2(G1[rp], __shfl_xor_sync(kFull, G1[rp], o));
          G2[rp] = add2(G2[rp], __shfl_xor_sync(kFull, G2[rp], o));
        }
      }
      float *accI = accR + ((rtb + I) * kTile) * kAcc3Stride + off;
#pragma unroll
      for (int rp = 0; rp < 4; ++rp) {
        if (rp == q) {
          const int r0 = p * 8 + 2 * rp;
          float s_lo, s_hi, g0l, g0h, g1l, g1h, g2l, g2h;
          upk(st[rp], s_lo, s_hi);
          upk(G0[rp], g0l, g0h);
          upk(G1[rp], g1l, g1h);
          upk(G2[rp], g2l, g2h);
          if (ROWS) {  // the record's only writer
            if ((int64_t)I * kTile + r0 < rcnt)
              *reinterpret_cast<float4 *>(accI + r0 * kAcc3Stride) =
                  make_float4(s_lo, g0l, g1l, g2l);
            if ((int64_t)I * kTile + r0 + 1 < rcnt)
              *reinterpret_cast<float4 *>(accI + (r0 + 1) * kAcc3Stride) =
                  make_float4(s_hi, g0h, g1h, g2h);
          } else {
            if ((int64_t)I * kTile + r0 < rcnt)
              red_add_v4(accI + r0 * kAcc3Stride, s_lo, g0l, g1l, g2l);
            if ((int64_t)I * kTile + r0 + 1 < rcnt)
              red_add_v4(accI + (r0 + 1) * kAcc3Stride, s_hi, g0h, g1h, g2h);
          }
        }
      }
    }
  }
}

}  // namespace ra
