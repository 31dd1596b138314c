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
// Roles (352 threads, one CTA per SM, persistent over the items):
//   warps 0-7  epilogue.  Warp w reads TMEM lanes 32 (w % 4) .. +31 (row =
//              lane) and columns [32 (w / 4), +32) of each S tile.  Per item
//              it turns each S tile into P; after the item's first tile it
//              writes the previous item's outputs (T into the per-point
//              records, the item's K) and starts copying the next item's rows,
//              which replace X once this item's last GEMM 1 has landed.
//   warp 8     lane 0 copies column tiles into a 4-stage shared-memory ring
//              (cp.async.bulk, no multicast, this GPU's memory only).
//   warp 9     lane 0 issues GEMM 1 of each tile into S stage t % 3 as soon
//              as its column tile has landed and the stage is free.
//   warp 10    lane 0 issues GEMM 2 of each tile as soon as its P is ready.
//              Two issuers, because tcgen05.mma issue is synchronous and a
//              barrier wait is slow: one issuer's waits are covered by the
//              other's MMAs.
// TMEM columns: X [0, DP) (hi in the first half, lo in the second, two fp16
// per column), T [DP, 2DP), three S/P stages of 64 columns from 2DP.  P (hi
// then lo, 16 columns each per 32-point half) overwrites the S columns its
// thread has already read.
//
// Every wait is bounded and gives up when another role has aborted; on expiry
// the kernel records kErrTimeout, drains what it issued, frees its TMEM and
// returns (the same contract as the other tensor-core kernels).
#pragma once

#include "ra_prep.cuh"
#include "ra_tcprim.cuh"

namespace ra {

constexpr int kT16Cols = 64;     // points per column tile
constexpr int kT16Stages = 4;    // column tiles in shared memory
constexpr int kT16EpiWarps = 8;
constexpr int kT16ProdWarp = 8;
constexpr int kT16MmaWarp = 9;    // GEMM 1 issuer
constexpr int kT16Mma2Warp = 10;  // GEMM 2 issuer
constexpr int kT16Threads = 352;
constexpr int kT16SlotFloats = 3 * kT16Cols;  // per tile: |x'|^2, |x'|^2 - log2 a, a 2^-f

__host__ __device__ constexpr int t16_tile_bytes(int DP) { return DP * 128; }  // hi or lo
__host__ __device__ constexpr int t16_stage_bytes(int DP) {
  return 2 * t16_tile_bytes(DP) + kT16SlotFloats * 4;
}
constexpr int kT16SStages = 3;   // S / P stages in TMEM
__host__ __device__ constexpr int t16_tmem_cols(int DP) {
  return 2 * DP + 64 * kT16SStages <= 256 ? 256 : 512;
}
constexpr int kT16Bars = 2 * kT16Stages + 3 * kT16SStages + 2;
__host__ __device__ constexpr size_t t16_smem_bytes(int DP) {
  // stages, the epilogue's row staging (2 DP bytes per thread), barriers,
  // TMEM address + abort flag, the epilogue's reductions
  return (size_t)kT16Stages * t16_stage_bytes(DP) + (size_t)32 * kT16EpiWarps * (2 * DP + 16) +
         kT16Bars * 8 + 16 + 2 * 128 * 8 * 2 + 2 * 8 * 8;
}
__host__ __device__ constexpr size_t t16_smem_request(int DP) {
  // at least 120 KB: one CTA per SM (each takes the TMEM columns it needs
  // for its whole persistent loop)
  return t16_smem_bytes(DP) > (size_t)120 * 1024 ? t16_smem_bytes(DP) : (size_t)120 * 1024;
}

// Everything a role needs about one work item, in one 64-byte record
// (t16_items_kernel), so that no role walks item -> pair -> metadata with
// dependent loads inside its loop.
struct ItemX {
  int64_t rbase;   // first point of the row cloud
  int64_t rcnt;    // points of the row cloud
  int64_t tb_row;  // first 64-point tile of the row cloud
  int64_t tb_col;  // first 64-point tile of the column cloud
  int32_t tile;    // 128-row tile of the item
  int32_t ntiles;  // 64-point column tiles
  int32_t flags;   // kIx* bits, block id << 4
  float cS;        // 2 / (2^e_row 2^e_col): 2 x'.y' from the scaled GEMM
  float lwsc;      // -f: log2 of the column weights' scale
  float tsc;       // 2^f / 2^e_col: T from the scaled GEMM
  float f2;        // 2^f
  int32_t pad;
};
static_assert(sizeof(ItemX) == 64, "one 64-byte record per item");
constexpr int kIxRowsX = 1, kIxColsX = 2, kIxSelf = 4, kIxFold = 8;

struct Tc16Args {
  const Item *items;
  const ItemX *ix;
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

// The ItemX records of all items (grid-stride over the device-side count).
template <int DP>
__global__ void __launch_bounds__(256) t16_items_kernel(const Item *items, const int64_t *n_items,
                                                         const Seg *seg, const double *meta_all,
                                                         const int64_t *tbase_x,
                                                         const int64_t *tbase_y, ItemX *ix) {
  const int64_t n = *n_items;
  for (int64_t it = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; it < n;
       it += (int64_t)gridDim.x * blockDim.x) {
    const Item item = items[it];
    const Seg sg = seg[item.pair];
    const int o = item.block;  // 0: x-y, 1: x-x, 2: y-y, 3: y-x
    const bool rows_x = (o == 0 || o == 1), cols_x = (o == 1 || o == 3);
    const int rside = rows_x ? 0 : 1, cside = cols_x ? 0 : 1;
    const double *meta = meta_all + item.pair * (int64_t)meta_stride(DP);
    const double csr = meta[meta_tc_cscale(DP) + rside], csc = meta[meta_tc_cscale(DP) + cside];
    const double wsc = meta[meta_tc_wscale(DP) + cside];
    ItemX x;
    x.rbase = rows_x ? sg.xs : sg.ys;
    x.rcnt = rows_x ? sg.xcount : sg.ycount;
    x.tb_row = (rows_x ? tbase_x : tbase_y)[item.pair];
    x.tb_col = (cols_x ? tbase_x : tbase_y)[item.pair];
    x.tile = item.tile;
    x.ntiles = (int32_t)ceil_div(cols_x ? sg.xcount : sg.ycount, (int64_t)kT16Cols);
    x.flags = (rows_x ? kIxRowsX : 0) | (cols_x ? kIxColsX : 0) | ((o == 1 || o == 2) ? kIxSelf : 0) |
              (meta[meta_tc_fold(DP) + cside] != 0.0 ? kIxFold : 0) | (o << 4);
    x.cS = (float)(2.0 / (csr * csc));
    x.lwsc = (float)log2(wsc);
    x.tsc = (float)(1.0 / (wsc * csc));
    x.f2 = (float)(1.0 / wsc);
    x.pad = 0;
    ix[it] = x;
  }
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}

template <int DP, int MODE>
__global__ void __launch_bounds__(kT16Threads, 1) tilestc16_kernel(Tc16Args A) {
  static_assert(DP == 32 || DP == 64 || DP == 128, "tensor-core path: DP in {32, 64, 128}");
  constexpr bool GRAD = MODE >= 1;
  constexpr bool SIG = MODE == 2;
  constexpr int NCOLS = t16_tmem_cols(DP);
  constexpr int C_T = DP, C_S = 2 * DP;  // X at [0, DP)
  constexpr int NS = kT16SStages;
  constexpr int TB = t16_tile_bytes(DP), SB = t16_stage_bytes(DP);
  constexpr uint32_t IDESC1 = t16_idesc(kT16Cols, 0), IDESC2 = t16_idesc(DP, 1);
  constexpr int ET = 32 * kT16EpiWarps;  // epilogue threads
  constexpr int NST = kT16Stages;
  constexpr int HC = DP / 4;  // TMEM cells per thread per X half (hi or lo)
  // staging bytes per epilogue thread: its half row (hi + lo chunks) on the
  // way into TMEM, or its half row of T on the way out; the 16-byte pad puts
  // consecutive threads' slots in different banks
  constexpr int XSB = 2 * DP + 16;

  extern __shared__ __align__(1024) uint8_t t16_smem[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(t16_smem + NST * SB + ET * XSB);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + kT16Bars);
  volatile int *abortf = reinterpret_cast<volatile int *>(tmem_slot + 1);
  double *red_s = reinterpret_cast<double *>(tmem_slot + 4);  // [2][128] row sums of half 1
  double *red_g = red_s + 256;                                // [2][128] sigma sums of half 1
  double *red_w = red_g + 256;                                // [2][8] per-warp K, S
  auto bar = [&](int i) { return smem_u32(bars + i); };
  // barrier ids: yfull[NST], yfree[NST], xfull, g1[NS], pfull[NS], g2[NS], tfree
  const int B_YFULL = 0, B_YFREE = NST, B_XFULL = 2 * NST, B_G1 = 2 * NST + 1,
            B_PFULL = 2 * NST + 1 + NS, B_G2 = 2 * NST + 1 + 2 * NS, B_TFREE = 2 * NST + 1 + 3 * NS;

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
    mbar_init(bar(B_XFULL), ET);
    for (int b = 0; b < NS; ++b) {
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

  if (warp < kT16EpiWarps) {
    // =========================== epilogue ===================================
    const int q = warp & 3, h = warp >> 2;
    const int r = 32 * q + lane;  // row within the item's 128-row tile
    const uint32_t tlane = tbase + ((uint32_t)(32 * q) << 16);
    // this thread's staging slot for its half of a row (hi chunks, lo chunks)
    const uint32_t xslot = smem_u32(t16_smem + NST * SB) + (uint32_t)(tid * XSB);
    // Row data of an item: the weight and |x'|^2 of this thread's row, and,
    // for an item with column tiles, its hi / lo chunks copied into the
    // staging slot (cp.async, zero-filled beyond the cloud).  Nothing here
    // waits: the loads land while the current item's tiles are processed.
    // X is committed (and `xfull` completes a phase) only for items with
    // column tiles, the items the MMA issuer waits for, so neither side can
    // run two phases ahead of the other.
    auto stage_rows = [&](const ItemX &I, float &a_out, float &xsq_out) {
      // the slot may still be the source of this thread's last T store
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      const bool rows_x = (I.flags & kIxRowsX) != 0;
      const int64_t row = (int64_t)I.tile * 128 + r;
      const int64_t sub = 2 * (int64_t)I.tile + (r >> 6);  // 64-point tile of this row
      const bool have = sub < ceil_div(I.rcnt, (int64_t)kT16Cols);
      const int64_t tile = I.tb_row + (have ? sub : 0);
      const int j = r & 63;
      a_out = row < I.rcnt ? (rows_x ? A.Ax : A.Ay)[I.rbase + row] : 0.f;
      xsq_out = have ? (rows_x ? A.cx : A.cy)[tile * kT16SlotFloats + j] : 0.f;
      if (I.ntiles == 0) return;  // no GEMM reads this item's rows
      const size_t off = (size_t)tile * TB + (size_t)((j >> 3) * 128 + (j & 7) * 16);
      const uint8_t *hs = (rows_x ? A.hx : A.hy) + off;
      const uint8_t *ls = (rows_x ? A.lx : A.ly) + off;
#pragma unroll
      for (int g = 0; g < DP / 16; ++g) {
        const int dg = h * (DP / 16) + g;  // coordinate group (8 coordinates, 16 bytes)
        cp_async16(xslot + 16 * g, hs + dg * 1024, have ? 16u : 0u);
        cp_async16(xslot + 16 * (DP / 16 + g), ls + dg * 1024, have ? 16u : 0u);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // the staged rows into X (this thread's lane, its half)
    auto commit_rows = [&]() {
      asm volatile("cp.async.wait_all;" ::: "memory");
      uint32_t ch[HC], cl[HC];
#pragma unroll
      for (int g = 0; g < DP / 16; ++g) {
        uint32_t v0, v1, v2, v3, w0, w1, w2, w3;
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(v0), "=r"(v1), "=r"(v2), "=r"(v3)
                     : "r"(xslot + 16 * g));
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3)
                     : "r"(xslot + 16 * (DP / 16 + g)));
        ch[4 * g] = v0; ch[4 * g + 1] = v1; ch[4 * g + 2] = v2; ch[4 * g + 3] = v3;
        cl[4 * g] = w0; cl[4 * g + 1] = w1; cl[4 * g + 2] = w2; cl[4 * g + 3] = w3;
      }
      tmem_st_n<HC>(tlane + h * HC, ch);           // hi: columns [0, DP/2)
      tmem_st_n<HC>(tlane + DP / 2 + h * HC, cl);  // lo: columns [DP/2, DP)
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      mbar_arrive(bar(B_XFULL));
    };

    // An item's outputs are written after the FIRST tile of the next item
    // (or after the loop): GEMM 2 of its last tile has landed by then, and
    // the tensor core has the next GEMM 1 while T is read out.
    struct Out {
      int64_t it, rbase, row;
      double s64, sg64;
      float a, tsc, f2;
      uint32_t tlast;  // the item's last column tile (if it has any)
      int flags, ntiles;
      bool rv;
    };
    bool ok = true;
    // all 256 threads, ok uniform: T into the records, the item's K and S
    auto outputs = [&](const Out &P, int rb) {
      const int o = P.flags >> 4;  // 0: x-y, 1: x-x, 2: y-y, 3: y-x
      const bool rows_x = (P.flags & kIxRowsX) != 0, self = (P.flags & kIxSelf) != 0;
      const bool crossb = (o == 0 || o == 3);
      if (h == 1) {
        red_s[rb * 128 + r] = P.s64;
        red_g[rb * 128 + r] = P.sg64;
      }
      if (GRAD && A.need_rows) {
        // this thread's half row of T: scaled into the staging slot, then one
        // bulk store of 2 DP bytes to its record (16-byte aligned: the record
        // stride is (2 DP + 4) floats).  The TMEM loads are warp-collective,
        // so every lane makes them; only rows inside the cloud store.
        const int toff = crossb ? DP : 0;
        constexpr int NW = DP / 2 < 32 ? DP / 2 : 32;
#pragma unroll
        for (int d0 = 0; d0 < DP / 2; d0 += NW) {
          float T[32];
          if (P.ntiles == 0) {
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
          if (P.rv) {
#pragma unroll
            for (int u = 0; u < NW; u += 4)
              asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(xslot + 4 * (d0 + u)),
                           "f"(T[u] * P.tsc), "f"(T[u + 1] * P.tsc), "f"(T[u + 2] * P.tsc),
                           "f"(T[u + 3] * P.tsc)
                           : "memory");
          }
        }
        if (P.rv) {
          float *dst = (rows_x ? A.accX : A.accY) + (P.rbase + P.row) * gen_acc_stride(DP);
          fence_async_smem();
          asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                           dst + toff + h * (DP / 2)),
                       "r"(xslot), "r"((uint32_t)(2 * DP))
                       : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
      if (GRAD && P.ntiles > 0) {
        tc_fence_before();
        mbar_arrive(bar(B_TFREE));  // T read: GEMM 2 of the next item may overwrite it
      }
      role_sync(1, ET);  // the half-1 sums are in red_s / red_g
      double kv = 0.0, sv = 0.0;
      if (h == 0) {
        const double f2 = (double)P.f2;
        const double sfull = (P.s64 + red_s[rb * 128 + r]) * f2;
        if (GRAD && A.need_rows && P.rv) {
          float *dst = (rows_x ? A.accX : A.accY) + (P.rbase + P.row) * gen_acc_stride(DP);
          dst[2 * DP + (crossb ? 1 : 0)] = (float)sfull;
        }
        // K (and S) partial of the item: a_i (s_i + [self] a_i), fixed order
        kv = (double)P.a * (sfull + (self ? (double)P.a : 0.0));
        sv = (double)P.a * (P.sg64 + red_g[rb * 128 + r]) * f2;
      }
      kv = warp_sum(kv);
      sv = warp_sum(sv);
      if (lane == 0 && h == 0) {
        red_w[rb * 8 + q] = kv;
        red_w[rb * 8 + 4 + q] = sv;
      }
      role_sync(1, ET);
      if (tid == 0) {
        const double K = red_w[rb * 8 + 0] + red_w[rb * 8 + 1] + red_w[rb * 8 + 2] + red_w[rb * 8 + 3];
        const double Sg = red_w[rb * 8 + 4] + red_w[rb * 8 + 5] + red_w[rb * 8 + 6] + red_w[rb * 8 + 7];
        A.itemK[P.it] = o == 3 ? 0.0 : K;
        A.itemS[P.it] = o == 3 ? 0.0 : Sg;
      }
    };
    // all 256 threads: wait for GEMM 2 of the item's last tile, agree, write
    auto finish = [&](const Out &P, int rb) {
      bool w = ok;
      if (ok && GRAD && P.ntiles > 0) {
        w = __all_sync(kFull, ws_wait(bar(B_G2 + (int)(P.tlast % NS)), (P.tlast / NS) & 1u,
                                      abortf, A.spin_limit));
        if (!w) fail();
      }
      if (role_sync_or(1, ET, !w)) ok = false;
      tc_fence_after();
      if (ok) outputs(P, rb);
    };

    uint32_t t = 0;  // column tiles seen (all items)
    int k = 0;       // items seen
    ItemX cur;
    float ca = 0.f, cxsq = 0.f;
    bool pending = false;
    Out prev;
    int prev_rb = 0;
    if (ifirst < n_items) {
      cur = A.ix[ifirst];
      stage_rows(cur, ca, cxsq);
      if (cur.ntiles > 0) commit_rows();
    }
    // Every warp runs the same sequence of named barriers whatever happens:
    // after a failed wait a warp skips the work but not the barriers, and
    // the agreements (bar.red.or) make `ok` uniform before any barrier that
    // only some paths would reach.
    for (int64_t it = ifirst; it < n_items; it += istep, ++k) {
      const bool has_next = it + istep < n_items;
      ItemX nxt;
      float na = 0.f, nxsq = 0.f;
      if (has_next) nxt = A.ix[it + istep];  // used after this item's first tile
      bool staged = false;
      const bool self = (cur.flags & kIxSelf) != 0, fold = (cur.flags & kIxFold) != 0;
      const int64_t row0 = (int64_t)cur.tile * 128;
      const int64_t row = row0 + r;
      const bool rv = row < cur.rcnt;
      const float a = ca, xsq = cxsq;
      const int ntiles = cur.ntiles;
      const float cS = cur.cS;
      const float nxf = -xsq + cur.lwsc;  // - |x'|^2 - f
      double s64 = 0.0, sg64 = 0.0;
      for (int jt = 0; jt < ntiles; ++jt, ++t) {
        const int ss = (int)(t % NS), ys = (int)(t % NST);
        if (ok) {
          // each warp waits for itself (warp-uniform outcome); a failed wait
          // records the abort at once, so the other warps' waits end too
          const bool w_ok = ws_wait(bar(B_YFULL + ys), (t / NST) & 1u, abortf, A.spin_limit) &&
                            ws_wait(bar(B_G1 + ss), (t / NS) & 1u, abortf, A.spin_limit);
          if (!__all_sync(kFull, w_ok)) {
            fail();
            ok = false;
          }
        }
        if (ok) {
          tc_fence_after();
          const float *cb = reinterpret_cast<const float *>(t16_smem + ys * SB + 2 * TB);
          const float *ysq = cb + 32 * h, *yq = cb + kT16Cols + 32 * h,
                      *bw = cb + 2 * kT16Cols + 32 * h;
          const int64_t j0 = (int64_t)jt * kT16Cols + 32 * h;
          const int64_t dj = row - j0;
          const int diag = (self && dj >= 0 && dj < 32) ? (int)dj : -1;
          // this warp's 32 columns meet the item's diagonal (warp-uniform)
          const bool dtile = self && j0 < row0 + 128 && row0 < j0 + 32;
          float S[32];
          tmem_ld32(tlane + C_S + 64 * ss + 32 * h, S);
          float st = 0.f, sgt = 0.f;
          uint32_t ph[16], pl[16];
          auto tile = [&](auto fold_t, auto diag_t) {
            constexpr bool FOLD = decltype(fold_t)::value, DG = decltype(diag_t)::value;
#pragma unroll
            for (int u2 = 0; u2 < 16; ++u2) {
              float wv[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int u = 2 * u2 + e;
                float w, r2 = 0.f;
                if (FOLD) {
                  w = ex2(fmaf(S[u], cS, nxf - yq[u]));
                  if (SIG) r2 = fmaxf(fmaf(-S[u], cS, xsq + ysq[u]), 0.f);
                } else {
                  r2 = fmaxf(fmaf(-S[u], cS, xsq + ysq[u]), 0.f);
                  w = bw[u] * ex2(-r2);
                }
                if (DG && u == diag) w = 0.f;
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
          };
          if (!fold)
            tile(BoolC<false>{}, BoolC<true>{});
          else if (dtile)
            tile(BoolC<true>{}, BoolC<true>{});
          else
            tile(BoolC<true>{}, BoolC<false>{});
          if (GRAD) {
            tmem_st16(tlane + C_S + 64 * ss + 32 * h, ph);
            tmem_st16(tlane + C_S + 64 * ss + 32 * h + 16, pl);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          }
          s64 += (double)st;
          if (SIG) sg64 += (double)sgt;
          tc_fence_before();
          mbar_arrive(bar(B_PFULL + ss));  // P ready, S and the slot values read
        }
        if (jt == 0 && pending) {
          finish(prev, prev_rb);  // the previous item's outputs
          pending = false;
        }
        if (ok && jt == 0 && has_next) {
          stage_rows(nxt, na, nxsq);  // the next item's rows, in flight during this item
          staged = true;
        }
      }
      if (ntiles == 0 && pending) {
        finish(prev, prev_rb);
        pending = false;
      }
      if (ok && has_next && !staged) stage_rows(nxt, na, nxsq);
      // every GEMM 1 of this item has landed (its S tiles were read): the next
      // item's rows replace X
      if (ok && has_next && nxt.ntiles > 0) commit_rows();
      if (role_sync_or(1, ET, !ok)) ok = false;  // one agreement per item
      if (!ok) break;
      prev.it = it;
      prev.rbase = cur.rbase;
      prev.row = row;
      prev.s64 = s64;
      prev.sg64 = sg64;
      prev.a = a;
      prev.tsc = cur.tsc;
      prev.f2 = cur.f2;
      prev.tlast = t - 1u;
      prev.flags = cur.flags;
      prev.ntiles = ntiles;
      prev.rv = rv;
      prev_rb = k & 1;
      pending = true;
      cur = nxt;
      ca = na;
      cxsq = nxsq;
    }
    if (pending) finish(prev, prev_rb);  // every thread: `pending` and the agreements are uniform
    asm volatile("cp.async.wait_all;" ::: "memory");  // no copy in flight at exit
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  } else if (warp == kT16ProdWarp) {
    // ====================== producer: column tiles ===========================
    uint32_t t = 0;
    uint32_t armed[NST];
#pragma unroll
    for (int s = 0; s < NST; ++s) armed[s] = 0;
    if (lane == 0) {
      for (int64_t it = ifirst; it < n_items && !*abortf; it += istep) {
        const ItemX I = A.ix[it];
        const bool cols_x = (I.flags & kIxColsX) != 0;
        const int ntiles = I.ntiles;
        const int64_t tb0 = I.tb_col;
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
  } else if (warp == kT16MmaWarp && lane == 0) {
    // ======================= GEMM 1 issuer ==================================
    // tcgen05.mma issue is synchronous (the tensor core queues only a few
    // instructions) and a barrier wait costs ~150 cycles even when it is
    // already satisfied, so each GEMM has its own issuing warp: one issuer's
    // waits are covered by the other's MMAs.  Ordering between the two goes
    // through the barriers: GEMM 1 of tile t waits for GEMM 2 of tile t - 3
    // (its S stage), GEMM 2 of tile t for the epilogue's P of tile t.
    uint32_t t = 0, m = 0, n_g1 = 0, last_g1 = 0;
    bool ok = true;
    for (int64_t it = ifirst; it < n_items && ok && !*abortf && !A.no_mma; it += istep) {
      const int ntiles = A.ix[it].ntiles;
      if (ntiles == 0) continue;
      // X holds this item's rows once the epilogue's m-th commit has landed
      // (one commit per item with column tiles)
      if (!ws_wait(bar(B_XFULL), m & 1u, abortf, A.spin_limit)) {
        ok = false;
        break;
      }
      for (int jt = 0; jt < ntiles; ++jt, ++t) {
        const int ss = (int)(t % NS), ys = (int)(t % NST);
        if (!ws_wait(bar(B_YFULL + ys), (t / NST) & 1u, abortf, A.spin_limit)) {
          ok = false;
          break;
        }
        // S stage ss is free once the tile NS back is fully consumed: its
        // GEMM 2 done (gradients) or its epilogue done (K only)
        if (t >= (uint32_t)NS) {
          const bool w = GRAD ? ws_wait(bar(B_G2 + ss), ((t / NS) - 1u) & 1u, abortf, A.spin_limit)
                              : ws_wait(bar(B_PFULL + ss), ((t / NS) - 1u) & 1u, abortf,
                                        A.spin_limit);
          if (!w) {
            ok = false;
            break;
          }
        }
        tc_fence_after();
        const uint32_t yh = smem_u32(t16_smem + ys * SB), yl = yh + TB;
        const uint32_t xh = tbase, xl = xh + DP / 2;
        const uint32_t d = tbase + C_S + 64 * ss;
#pragma unroll
        for (int kk = 0; kk < DP / 16; ++kk) {
          const uint64_t bh = tc_desc(yh + kk * 2048, 1024, 128);
          const uint64_t bl = tc_desc(yl + kk * 2048, 1024, 128);
          t16_mma(d, xh + 8 * kk, bh, IDESC1, kk > 0 ? 1u : 0u);
          t16_mma(d, xh + 8 * kk, bl, IDESC1, 1u);
          t16_mma(d, xl + 8 * kk, bh, IDESC1, 1u);
        }
        tc_commit(bar(B_G1 + ss));
        ++n_g1;
        last_g1 = t;
      }
      ++m;
    }
    if (!ok) fail();
    // every MMA this thread issued has landed before TMEM is freed (bounded)
    if (n_g1 > 0) (void)mbar_wait(bar(B_G1 + (int)(last_g1 % NS)), (last_g1 / NS) & 1u);
  } else if (warp == kT16Mma2Warp && lane == 0) {
    // ======================= GEMM 2 issuer ==================================
    uint32_t t = 0, m = 0, n_g2 = 0, last_g2 = 0;
    bool ok = true;
    for (int64_t it = ifirst; it < n_items && ok && !*abortf && !A.no_mma; it += istep) {
      const int ntiles = A.ix[it].ntiles;
      if (ntiles == 0) continue;
      for (int jt = 0; jt < ntiles; ++jt, ++t) {
        const int ss = (int)(t % NS), ys = (int)(t % NST);
        if (!ws_wait(bar(B_PFULL + ss), (t / NS) & 1u, abortf, A.spin_limit)) {
          ok = false;
          break;
        }
        // the item's first GEMM 2 overwrites T: the previous item's T read
        if (GRAD && jt == 0 && m > 0 &&
            !ws_wait(bar(B_TFREE), (m - 1u) & 1u, abortf, A.spin_limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (GRAD) {
          const uint32_t yh = smem_u32(t16_smem + ys * SB), yl = yh + TB;
#pragma unroll
          for (int kk = 0; kk < kT16Cols / 16; ++kk) {
            const uint32_t pa = tbase + C_S + 64 * ss + 32 * (kk >> 1) + 8 * (kk & 1);
            const uint64_t bh = tc_desc(yh + kk * 256, 128, 1024);
            const uint64_t bl = tc_desc(yl + kk * 256, 128, 1024);
            t16_mma(tbase + C_T, pa, bh, IDESC2, (jt == 0 && kk == 0) ? 0u : 1u);
            t16_mma(tbase + C_T, pa, bl, IDESC2, 1u);
            t16_mma(tbase + C_T, pa + 16, bh, IDESC2, 1u);
          }
          tc_commit(bar(B_G2 + ss));
          tc_commit(bar(B_YFREE + ys));
          ++n_g2;
          last_g2 = t;
        } else {
          // K only: the stage's slot values were read by the epilogue
          mbar_arrive(bar(B_YFREE + ys));
        }
      }
      ++m;
    }
    if (!ok) fail();
    if (n_g2 > 0) (void)mbar_wait(bar(B_G2 + (int)(last_g2 % NS)), (last_g2 / NS) & 1u);
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
