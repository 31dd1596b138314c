// ra_tc16.cuh -- tensor-core kernel of the generic layout for padded widths
// DP in {32, 64, 128} (the high-dimensional embedding case).
//
// Work items are those of the SIMT kernel (ra_tilesg.cuh): (pair,
// orientation, 128-row tile), rows-only, every orientation evaluated, so each
// point's record has one writer.  Per column tile of 64 points, with x', y'
// the pre-scaled coordinates (k = 2^-|x'-y'|^2):
//   GEMM 1  S = X Y^T                 (M = 128 rows, N = 64 points, K = DP)
//   epilogue w = b_j 2^-(|x'|^2 + |y'|^2 - 2 S)  (the diagonal left out in
//           self blocks), row sums in registers, P = w into TMEM
//   GEMM 2  T += P Y                  (M = 128 rows, N = DP, K = 64 points)
// Both GEMMs are tcgen05.mma kind::f16 with fp32 accumulation and three
// products per GEMM (a = a_hi + a_lo in fp16: hi*hi + hi*lo + lo*hi), which
// carries ~22 significant bits, as 3xTF32 does, at twice the tf32 rate and
// with half the operand bytes.  fp16 has a narrow exponent range, so every
// operand is scaled by a power of two chosen per pair side from a bound on
// its magnitude (the coordinates to at most 2^15, the weights into (1/2, 1]);
// the scales are exact and are undone in the epilogue.
//
// Data (written by packtc_kernel, ra_prep.cuh): each cloud in 64-point tiles
// of fp16 hi and lo arrays in the canonical no-swizzle core-matrix layout,
//     byte offset of (point j, coordinate d) = (d/8)*1024 + (j/8)*128
//                                              + (j%8)*16 + (d%8)*2,
// and per slot |x'|^2, |x'|^2 - log2 a and a 2^-f (a: normalised weight).
// One copy of a tile in shared memory is GEMM 1's K-major B operand (N =
// point, K = coordinate: leading byte offset 1024 between coordinate groups,
// stride byte offset 128 between point groups) and GEMM 2's MN-major B
// operand (N = coordinate, K = point: leading byte offset 128 between point
// groups, stride byte offset 1024 between coordinate groups).
//
// Roles (320 threads, one CTA per SM, persistent over the items):
//   warps 0-7  epilogue.  Warp w reads TMEM lanes 32 (w % 4) .. +31 (row =
//              lane) and columns [32 (w / 4), +32) of each S tile.  Per item
//              it first writes the NEXT item's rows (hi/lo) into the other X
//              buffer, then turns each S tile into P, and at the end of the
//              item reads T and writes the per-point records.
//   warp 8     lane 0 copies column tiles into a 4-stage shared-memory ring
//              (cp.async.bulk, no multicast, this GPU's memory only).
//   warp 9     lane 0 issues the MMAs: GEMM 1 of tile t into S stage t % 2,
//              then GEMM 2 of tile t - 1, so the tensor core has GEMM 1 of
//              the next tile while the epilogue works on the current one.
// TMEM columns: X buffers [0, DP) and [DP, 2DP) (hi in the first half, lo in
// the second, two fp16 per column), T [2DP, 3DP), S/P stages [3DP, 3DP+64)
// and [3DP+64, 3DP+128).  P (hi then lo, 16 columns each per 32-point half)
// overwrites the S columns its thread has already read.
//
// Every wait is bounded and gives up when another role has aborted; on expiry
// the kernel records kErrTimeout, drains what it issued, frees its TMEM and
// returns (the same contract as the other tensor-core kernels).
#pragma once

#include "ra_tcws.cuh"

namespace ra {

constexpr int kT16Cols = 64;     // points per column tile
constexpr int kT16Stages = 4;    // column tiles in shared memory
constexpr int kT16EpiWarps = 8;
constexpr int kT16ProdWarp = 8;
constexpr int kT16MmaWarp = 9;
constexpr int kT16Threads = 320;
constexpr int kT16SlotFloats = 3 * kT16Cols;  // per tile: |x'|^2, |x'|^2 - log2 a, a 2^-f

__host__ __device__ constexpr int t16_tile_bytes(int DP) { return DP * 128; }  // hi or lo
__host__ __device__ constexpr int t16_stage_bytes(int DP) {
  return 2 * t16_tile_bytes(DP) + kT16SlotFloats * 4;
}
__host__ __device__ constexpr int t16_tmem_cols(int DP) { return 3 * DP + 128 <= 256 ? 256 : 512; }
constexpr int kT16Bars = 2 * kT16Stages + 9;
__host__ __device__ constexpr size_t t16_smem_bytes(int DP) {
  // stages, barriers, TMEM address + abort flag, the epilogue's reductions
  return (size_t)kT16Stages * t16_stage_bytes(DP) + kT16Bars * 8 + 16 + 128 * 8 * 2 + 16 * 8;
}
__host__ __device__ constexpr size_t t16_smem_request(int DP) {
  // at least 120 KB: one CTA per SM (each takes the TMEM columns it needs
  // for its whole persistent loop)
  return t16_smem_bytes(DP) > (size_t)120 * 1024 ? t16_smem_bytes(DP) : (size_t)120 * 1024;
}

struct Tc16Args {
  const Item *items;
  const int64_t *n_items;
  const Seg *seg;
  const double *meta;                   // per pair (meta_tc_* scales)
  const int64_t *tbase_x, *tbase_y;     // first 64-point tile of each pair's cloud
  const uint8_t *hx, *hy, *lx, *ly;     // fp16 hi / lo tiles
  const float *cx, *cy;                 // per tile: kT16SlotFloats slot values
  const float *Ax, *Ay;                 // [num] normalised weights (rows)
  float *accX, *accY;                   // [num][gen_acc_stride(DP)]
  double *itemK, *itemS;
  int need_rows;
  int shard_index, shard_count;
  int *err;
  unsigned spin_limit;
  int no_mma;
};

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes,
                                         uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(mbar)
      : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mbar), "r"(bytes)
               : "memory");
}
__host__ __device__ constexpr uint32_t t16_idesc(int N, int b_major) {
  // D f32, A and B f16, A K-major, B K-major (0) or MN-major (1), M = 128
  return (1u << 4) | ((uint32_t)b_major << 16) | ((uint32_t)(N >> 3) << 17) | (8u << 24);
}
__device__ __forceinline__ void t16_mma(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  const uint32_t zero = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(zero));
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(
                   taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
               "r"(r[7])
               : "memory");
}
template <int N>
__device__ __forceinline__ void tmem_st_n(uint32_t taddr, const uint32_t (&r)[N]) {
  static_assert(N == 8 || N == 16 || N == 32, "tcgen05.st width");
  if constexpr (N == 8) tmem_st8(taddr, r);
  else if constexpr (N == 16) tmem_st16(taddr, r);
  else tmem_st32(taddr, r);
}
// two floats -> one cell of two fp16 (lo -> bits 0-15, hi -> bits 16-31)
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

template <int DP, int MODE>
__global__ void __launch_bounds__(kT16Threads, 1) tilestc16_kernel(Tc16Args A) {
  static_assert(DP == 32 || DP == 64 || DP == 128, "tensor-core path: DP in {32, 64, 128}");
  constexpr bool GRAD = MODE >= 1;
  constexpr bool SIG = MODE == 2;
  constexpr int NCOLS = t16_tmem_cols(DP);
  constexpr int C_T = 2 * DP, C_S = 3 * DP;
  constexpr int TB = t16_tile_bytes(DP), SB = t16_stage_bytes(DP);
  constexpr uint32_t IDESC1 = t16_idesc(kT16Cols, 0), IDESC2 = t16_idesc(DP, 1);
  constexpr int ET = 32 * kT16EpiWarps;  // epilogue threads
  constexpr int NST = kT16Stages;
  constexpr int HC = DP / 4;  // TMEM cells per thread per X half (hi or lo)

  extern __shared__ __align__(1024) uint8_t t16_smem[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(t16_smem + NST * SB);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + kT16Bars);
  volatile int *abortf = reinterpret_cast<volatile int *>(tmem_slot + 1);
  double *red_s = reinterpret_cast<double *>(tmem_slot + 4);  // [128] row sums of half 1
  double *red_g = red_s + 128;                                // [128] sigma sums of half 1
  double *red_w = red_g + 128;                                // [16] per-warp K, S
  auto bar = [&](int i) { return smem_u32(bars + i); };
  // barrier ids: yfull[s], yfree[s], xfull[2], g1[2], pfull[2], g2[2], tfree
  const int B_YFULL = 0, B_YFREE = NST, B_XFULL = 2 * NST, B_G1 = 2 * NST + 2,
            B_PFULL = 2 * NST + 4, B_G2 = 2 * NST + 6, B_TFREE = 2 * NST + 8;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(NCOLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(bar(B_YFULL + s), 1);
      mbar_init(bar(B_YFREE + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(B_XFULL + b), ET);
      mbar_init(bar(B_G1 + b), 1);
      mbar_init(bar(B_PFULL + b), ET);
      mbar_init(bar(B_G2 + b), 1);
    }
    mbar_init(bar(B_TFREE), ET);
    *abortf = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  const int64_t n_items = *A.n_items;
  const int64_t istep = (int64_t)gridDim.x * A.shard_count;
  const int64_t ifirst = (int64_t)blockIdx.x * A.shard_count + A.shard_index;
  auto fail = [&]() {
    if (!*abortf) {
      *abortf = 1;
      atomicOr(A.err, (int)kErrTimeout);
    }
  };
  // column tiles of an item
  auto item_tiles = [&](const Item &item, const Seg &sg) {
    const bool cols_x = (item.block == 1 || item.block == 3);
    return (int)ceil_div(cols_x ? sg.xcount : sg.ycount, (int64_t)kT16Cols);
  };

  if (warp < kT16EpiWarps) {
    // =========================== epilogue ===================================
    const int q = warp & 3, h = warp >> 2;
    const int r = 32 * q + lane;  // row within the item's 128-row tile
    const uint32_t tlane = tbase + ((uint32_t)(32 * q) << 16);
    // this thread's half of the next item's rows (hi, lo) into X buffer b
    auto load_x = [&](int64_t it, int b) {
      const Item item = A.items[it];
      const Seg sg = A.seg[item.pair];
      const bool rows_x = (item.block == 0 || item.block == 1);
      const int64_t rcnt = rows_x ? sg.xcount : sg.ycount;
      const int64_t sub = 2 * (int64_t)item.tile + (r >> 6);  // 64-point tile of this row
      const bool have = sub < ceil_div(rcnt, (int64_t)kT16Cols);
      const int64_t tile = (rows_x ? A.tbase_x : A.tbase_y)[item.pair] + sub;
      const int j = r & 63;
      const size_t off = (size_t)tile * TB + (size_t)((j >> 3) * 128 + (j & 7) * 16);
      const uint8_t *hs = (rows_x ? A.hx : A.hy) + off;
      const uint8_t *ls = (rows_x ? A.lx : A.ly) + off;
      uint32_t ch[HC], cl[HC];
#pragma unroll
      for (int g = 0; g < DP / 16; ++g) {
        const int dg = h * (DP / 16) + g;  // coordinate group (8 coordinates, 16 bytes)
        uint4 vh = make_uint4(0u, 0u, 0u, 0u), vl = vh;
        if (have) {
          vh = *reinterpret_cast<const uint4 *>(hs + dg * 1024);
          vl = *reinterpret_cast<const uint4 *>(ls + dg * 1024);
        }
        ch[4 * g] = vh.x; ch[4 * g + 1] = vh.y; ch[4 * g + 2] = vh.z; ch[4 * g + 3] = vh.w;
        cl[4 * g] = vl.x; cl[4 * g + 1] = vl.y; cl[4 * g + 2] = vl.z; cl[4 * g + 3] = vl.w;
      }
      const uint32_t cx = (uint32_t)(b * DP);
      tmem_st_n<HC>(tlane + cx + h * HC, ch);           // hi: columns [cx, cx + DP/2)
      tmem_st_n<HC>(tlane + cx + DP / 2 + h * HC, cl);  // lo: columns [cx + DP/2, cx + DP)
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      mbar_arrive(bar(B_XFULL + b));
    };

    uint32_t t = 0;  // column tiles seen (all items)
    int k = 0;       // items seen
    if (ifirst < n_items) load_x(ifirst, 0);
    for (int64_t it = ifirst; it < n_items; it += istep, ++k) {
      if (it + istep < n_items) load_x(it + istep, (k + 1) & 1);
      const Item item = A.items[it];
      const Seg sg = A.seg[item.pair];
      const int o = item.block;  // 0: x-y, 1: x-x, 2: y-y, 3: y-x
      const bool rows_x = (o == 0 || o == 1), cols_x = (o == 1 || o == 3);
      const bool self = (o == 1 || o == 2);
      const int rside = rows_x ? 0 : 1, cside = cols_x ? 0 : 1;
      const int64_t rbase = rows_x ? sg.xs : sg.ys, rcnt = rows_x ? sg.xcount : sg.ycount;
      const int64_t row0 = (int64_t)item.tile * 128;
      const int64_t row = row0 + r;
      const bool rv = row < rcnt;
      const float a = rv ? (rows_x ? A.Ax : A.Ay)[rbase + row] : 0.f;
      const int ntiles = item_tiles(item, sg);
      // |x'|^2 of this row (packed slot value; 0 beyond the cloud)
      float xsq = 0.f;
      {
        const int64_t sub = 2 * (int64_t)item.tile + (r >> 6);
        if (sub < ceil_div(rcnt, (int64_t)kT16Cols))
          xsq = (rows_x ? A.cx : A.cy)[((rows_x ? A.tbase_x : A.tbase_y)[item.pair] + sub) *
                                           kT16SlotFloats + (r & 63)];
      }
      const double *meta = A.meta + item.pair * (int64_t)meta_stride(DP);
      const double csr = meta[meta_tc_cscale(DP) + rside], csc = meta[meta_tc_cscale(DP) + cside];
      const double wsc = meta[meta_tc_wscale(DP) + cside];  // 2^-f of the column weights
      const bool fold = meta[meta_tc_fold(DP) + cside] != 0.0;
      const float cS = (float)(2.0 / (csr * csc));      // 2 S = cS S'
      const float nxf = -xsq + (float)log2(wsc);        // - |x'|^2 - f
      float sr = 0.f;
      double s64 = 0.0, sg64 = 0.0;
      bool ok = true;
      for (int jt = 0; jt < ntiles; ++jt, ++t) {
        const int ss = (int)(t & 1u), ys = (int)(t % NST);
        const bool w_ok = ws_wait(bar(B_YFULL + ys), (t / NST) & 1u, abortf, A.spin_limit) &&
                          ws_wait(bar(B_G1 + ss), (t >> 1) & 1u, abortf, A.spin_limit);
        if (role_sync_or(1, ET, !w_ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float *cb = reinterpret_cast<const float *>(t16_smem + ys * SB + 2 * TB);
        const float *ysq = cb, *yq = cb + kT16Cols, *bw = cb + 2 * kT16Cols;
        const int64_t j0 = (int64_t)jt * kT16Cols + 32 * h;
        const int64_t dj = row - j0;
        const int diag = (self && dj >= 0 && dj < 32) ? (int)dj : -1;
        float S[32];
        tmem_ld32(tlane + C_S + 64 * ss + 32 * h, S);
        float st = 0.f, sgt = 0.f;
        uint32_t ph[16], pl[16];
#pragma unroll
        for (int u2 = 0; u2 < 16; ++u2) {
          float wv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int u = 2 * u2 + e, j = 32 * h + u;
            float w, r2 = 0.f;
            if (fold) {
              w = ex2(fmaf(S[u], cS, nxf - yq[j]));
              if (SIG) r2 = fmaxf(fmaf(-S[u], cS, xsq + ysq[j]), 0.f);
            } else {
              r2 = fmaxf(fmaf(-S[u], cS, xsq + ysq[j]), 0.f);
              w = bw[j] * ex2(-r2);
            }
            if (u == diag) w = 0.f;
            st += w;
            if (SIG) sgt = fmaf(w, r2, sgt);
            wv[e] = w;
          }
          if (GRAD) {
            const float h0 = __uint_as_float(__float_as_uint(wv[0]) & 0xFFFFE000u);
            const float h1 = __uint_as_float(__float_as_uint(wv[1]) & 0xFFFFE000u);
            ph[u2] = pack_f16x2(h0, h1);
            pl[u2] = pack_f16x2(wv[0] - h0, wv[1] - h1);
          }
        }
        if (GRAD) {
          tmem_st16(tlane + C_S + 64 * ss + 32 * h, ph);
          tmem_st16(tlane + C_S + 64 * ss + 32 * h + 16, pl);
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        sr += st;
        s64 += (double)st;
        if (SIG) sg64 += (double)sgt;
        tc_fence_before();
        mbar_arrive(bar(B_PFULL + ss));  // P ready, S and the slot values read
      }
      (void)sr;
      if (ok && GRAD && ntiles > 0) {
        // T of the item: after GEMM 2 of its last tile
        const uint32_t tl = t - 1u;
        const bool w_ok = ws_wait(bar(B_G2 + (int)(tl & 1u)), (tl >> 1) & 1u, abortf, A.spin_limit);
        if (role_sync_or(1, ET, !w_ok)) ok = false;
        tc_fence_after();
      }
      if (!ok) {
        fail();
        break;
      }
      const double f2 = 1.0 / wsc;  // 2^f
      // ---- item outputs -------------------------------------------------------
      if (GRAD && A.need_rows) {
        float *dst = (rows_x ? A.accX : A.accY) + (rbase + row) * gen_acc_stride(DP);
        const bool crossb = (o == 0 || o == 3);
        const int toff = crossb ? DP : 0, soff = 2 * DP + (crossb ? 1 : 0);
        const float tsc = (float)(f2 / csc);  // T = T' 2^f / 2^e
#pragma unroll
        for (int d0 = 0; d0 < DP / 2; d0 += (DP / 2 < 32 ? DP / 2 : 32)) {
          constexpr int NW = DP / 2 < 32 ? DP / 2 : 32;
          float T[32];
          if (ntiles == 0) {
#pragma unroll
            for (int u = 0; u < 32; ++u) T[u] = 0.f;
          } else if (NW == 32) {
            tmem_ld32(tlane + C_T + h * (DP / 2) + d0, T);
          } else {
            float T16[16];
            tmem_ld16(tlane + C_T + h * (DP / 2) + d0, T16);
#pragma unroll
            for (int u = 0; u < 16; ++u) T[u] = T16[u];
          }
          if (rv) {
#pragma unroll
            for (int u = 0; u < NW; u += 4)
              *reinterpret_cast<float4 *>(dst + toff + h * (DP / 2) + d0 + u) =
                  make_float4(T[u] * tsc, T[u + 1] * tsc, T[u + 2] * tsc, T[u + 3] * tsc);
          }
        }
        // the row's total over both halves, in a fixed order
        if (h == 1) red_s[r] = s64;
        role_sync(1, ET);
        if (h == 0 && rv) dst[soff] = (float)((s64 + red_s[r]) * f2);
        role_sync(1, ET);
      }
      if (GRAD && ntiles > 0) {
        tc_fence_before();
        mbar_arrive(bar(B_TFREE));  // T read: GEMM 2 of the next item may overwrite it
      }
      // K (and S) partial of the item: a_i (s_i + [self] a_i), fixed order
      if (h == 1) {
        red_s[r] = s64;
        red_g[r] = sg64;
      }
      role_sync(1, ET);
      double kv = 0.0, sv = 0.0;
      if (h == 0) {
        const double sfull = (s64 + red_s[r]) * f2;
        kv = (double)a * (sfull + (self ? (double)a : 0.0));
        sv = (double)a * (sg64 + red_g[r]) * f2;
      }
      kv = warp_sum(kv);
      sv = warp_sum(sv);
      if (lane == 0 && h == 0) {
        red_w[q] = kv;
        red_w[4 + q] = sv;
      }
      role_sync(1, ET);
      if (tid == 0) {
        const double K = red_w[0] + red_w[1] + red_w[2] + red_w[3];
        const double Sg = red_w[4] + red_w[5] + red_w[6] + red_w[7];
        A.itemK[it] = o == 3 ? 0.0 : K;
        A.itemS[it] = o == 3 ? 0.0 : Sg;
      }
      role_sync(1, ET);  // red_* are rewritten by the next item
    }
  } else if (warp == kT16ProdWarp) {
    // ====================== producer: column tiles ===========================
    uint32_t t = 0;
    uint32_t armed[NST];
#pragma unroll
    for (int s = 0; s < NST; ++s) armed[s] = 0;
    if (lane == 0) {
      for (int64_t it = ifirst; it < n_items && !*abortf; it += istep) {
        const Item item = A.items[it];
        const Seg sg = A.seg[item.pair];
        const bool cols_x = (item.block == 1 || item.block == 3);
        const int ntiles = item_tiles(item, sg);
        const int64_t tb0 = (cols_x ? A.tbase_x : A.tbase_y)[item.pair];
        const uint8_t *hs = cols_x ? A.hx : A.hy, *ls = cols_x ? A.lx : A.ly;
        const float *cs = cols_x ? A.cx : A.cy;
        bool ok = true;
        for (int jt = 0; jt < ntiles; ++jt, ++t) {
          const int s = (int)(t % NST);
          if (t >= (uint32_t)NST &&
              !ws_wait(bar(B_YFREE + s), ((t / NST) - 1u) & 1u, abortf, A.spin_limit)) {
            ok = false;
            break;
          }
          const int64_t tile = tb0 + jt;
          const uint32_t dst = smem_u32(t16_smem + s * SB);
          mbar_expect_tx(bar(B_YFULL + s), (uint32_t)SB);
          bulk_g2s(dst, hs + (size_t)tile * TB, (uint32_t)TB, bar(B_YFULL + s));
          bulk_g2s(dst + TB, ls + (size_t)tile * TB, (uint32_t)TB, bar(B_YFULL + s));
          bulk_g2s(dst + 2 * TB, cs + tile * kT16SlotFloats, (uint32_t)(kT16SlotFloats * 4),
                   bar(B_YFULL + s));
          ++armed[s];
        }
        if (!ok) {
          fail();
          break;
        }
      }
      // every copy issued has landed before the CTA can exit (bounded)
#pragma unroll
      for (int s = 0; s < NST; ++s)
        if (armed[s] > 0) (void)mbar_wait(bar(B_YFULL + s), (armed[s] - 1u) & 1u);
    }
  } else if (lane == 0) {
    // ============================ MMA issuer =================================
    uint32_t t = 0;           // column tiles (all items)
    uint32_t m = 0;           // items with column tiles
    uint32_t n_g1 = 0, n_g2 = 0;
    uint32_t last_g1 = 0, last_g2 = 0;
    bool ok = true;
    // pending GEMM 2: the previous tile's
    bool pend = false;
    uint32_t p_t = 0, p_m = 0;
    bool p_first = false;
    auto issue_g2 = [&]() -> bool {
      const int ss = (int)(p_t & 1u), ys = (int)(p_t % NST);
      if (!ws_wait(bar(B_PFULL + ss), (p_t >> 1) & 1u, abortf, A.spin_limit)) return false;
      if (GRAD && p_first && p_m > 0 &&
          !ws_wait(bar(B_TFREE), (p_m - 1u) & 1u, abortf, A.spin_limit))
        return false;
      tc_fence_after();
      if (GRAD) {
        const uint32_t yh = smem_u32(t16_smem + ys * SB), yl = yh + TB;
#pragma unroll
        for (int kk = 0; kk < kT16Cols / 16; ++kk) {
          const uint32_t pa = tbase + C_S + 64 * ss + 32 * (kk >> 1) + 8 * (kk & 1);
          const uint64_t bh = tc_desc(yh + kk * 256, 128, 1024);
          const uint64_t bl = tc_desc(yl + kk * 256, 128, 1024);
          t16_mma(tbase + C_T, pa, bh, IDESC2, (p_first && kk == 0) ? 0u : 1u);
          t16_mma(tbase + C_T, pa, bl, IDESC2, 1u);
          t16_mma(tbase + C_T, pa + 16, bh, IDESC2, 1u);
        }
        tc_commit(bar(B_G2 + ss));
        tc_commit(bar(B_YFREE + ys));
        ++n_g2;
        last_g2 = p_t;
      } else {
        // K only: the stage's slot values were read by the epilogue
        mbar_arrive(bar(B_YFREE + ys));
      }
      pend = false;
      return true;
    };
    int k = 0;
    for (int64_t it = ifirst; it < n_items && ok && !*abortf && !A.no_mma; it += istep, ++k) {
      const Item item = A.items[it];
      const Seg sg = A.seg[item.pair];
      const int ntiles = item_tiles(item, sg);
      if (ntiles == 0) continue;
      const int xb = k & 1;
      if (!ws_wait(bar(B_XFULL + xb), ((uint32_t)k >> 1) & 1u, abortf, A.spin_limit)) {
        ok = false;
        break;
      }
      for (int jt = 0; jt < ntiles; ++jt, ++t) {
        const int ss = (int)(t & 1u), ys = (int)(t % NST);
        if (!ws_wait(bar(B_YFULL + ys), (t / NST) & 1u, abortf, A.spin_limit)) {
          ok = false;
          break;
        }
        // S stage ss is free once the tile two back is fully consumed: its
        // GEMM 2 done (gradients) or its epilogue done (K only)
        if (t >= 2u) {
          const bool w = GRAD ? ws_wait(bar(B_G2 + ss), ((t >> 1) - 1u) & 1u, abortf, A.spin_limit)
                              : ws_wait(bar(B_PFULL + ss), ((t >> 1) - 1u) & 1u, abortf,
                                        A.spin_limit);
          if (!w) {
            ok = false;
            break;
          }
        }
        tc_fence_after();
        {
          const uint32_t yh = smem_u32(t16_smem + ys * SB), yl = yh + TB;
          const uint32_t xh = tbase + (uint32_t)(xb * DP), xl = xh + DP / 2;
#pragma unroll
          for (int kk = 0; kk < DP / 16; ++kk) {
            const uint64_t bh = tc_desc(yh + kk * 2048, 1024, 128);
            const uint64_t bl = tc_desc(yl + kk * 2048, 1024, 128);
            const uint32_t d = tbase + C_S + 64 * ss;
            t16_mma(d, xh + 8 * kk, bh, IDESC1, kk > 0 ? 1u : 0u);
            t16_mma(d, xh + 8 * kk, bl, IDESC1, 1u);
            t16_mma(d, xl + 8 * kk, bh, IDESC1, 1u);
          }
          tc_commit(bar(B_G1 + ss));
          ++n_g1;
          last_g1 = t;
        }
        if (pend && !issue_g2()) {
          ok = false;
          break;
        }
        pend = true;
        p_t = t;
        p_m = m;
        p_first = jt == 0;
      }
      ++m;
    }
    if (ok && pend && !*abortf && !issue_g2()) ok = false;
    if (!ok) fail();
    // every MMA issued has landed before TMEM is freed (bounded)
    if (n_g1 > 0) (void)mbar_wait(bar(B_G1 + (int)(last_g1 & 1u)), (last_g1 >> 1) & 1u);
    if (n_g2 > 0) (void)mbar_wait(bar(B_G2 + (int)(last_g2 & 1u)), (last_g2 >> 1) & 1u);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase),
                 "r"(NCOLS)
                 : "memory");
}

}  // namespace ra
