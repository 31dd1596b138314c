// ra_tc.cuh -- tensor-core (tcgen05) path of the generic layout, for padded
// dimensions DP in {32, 64, 128} (the high-dimensional embedding case).
//
// Same work items and outputs as tilesg_kernel (ra_tilesg.cuh): one CTA of
// 128 threads takes an item (pair, orientation, 128-row tile) and streams the
// column cloud in tiles of 64 points.  Thread t owns row t, which is also
// TMEM lane t, so every per-row quantity is reduced in registers.
//
// Per column tile, with x', y' the pre-scaled coordinates (k = 2^-|x'-y'|^2):
//   GEMM 1 (tcgen05.mma kind::tf32, A = X from TMEM, B = Y from smem):
//       S = X Y^T, 3xTF32 (x = x_hi + x_lo; S = hi*hi + hi*lo + lo*hi), so S
//       keeps ~fp32 accuracy; plain TF32 would put a 1e-3 relative error on
//       r^2 = |x'|^2 + |y'|^2 - 2 S.
//   epilogue (registers): w = b_j 2^(-r^2) (diagonal left out in self
//       blocks), row sums s_i = sum w, S_i = sum w r^2, and P = w split into
//       tf32 hi/lo and stored back into TMEM.  With the tile's weights all
//       >= 0 the weight is folded into the exponent: w = 2^(2S - |x'|^2 -
//       (|y'|^2 - log2 b_j)), one FADD + one FFMA + EX2 per term; P's hi half
//       is w with the low 13 mantissa bits cleared (exact in tf32) and lo the
//       exact remainder.
//   GEMM 2 (A = P from TMEM, B = the Y tile stored transposed):
//       T_i += sum_j w_ij y'_j, again 3xTF32, accumulated in TMEM over all
//       column tiles of the item.
// The epilogue kernel forms G_i = x'_i s_i - T_i exactly as for tilesg.
//
// TMEM columns (512 at DP = 128): X_hi [0, DP), X_lo [DP, 2DP), S / P_hi
// [2DP, 2DP+64), P_lo [2DP+64, 2DP+128), T [2DP+128, 3DP+128).
// Shared memory, canonical no-swizzle K-major operands (core matrix = 8 rows
// x 16 bytes): Y_hi, Y_lo for GEMM 1 (N = point j, K = coordinate d), chunk
// (j, coordinates 4c..4c+3) at c * 1024 + j * 16; and the transposes Yt_hi,
// Yt_lo for GEMM 2 (N = d, K = j), chunk (d, points 4q..4q+3) at
// (d / 8) * 2048 + q * 128 + (d % 8) * 16.  (An MN-major tf32 operand would
// need the 128-byte/32-byte-atom swizzle; the plain transposed copy is
// simpler and costs 64 KB of shared memory at DP = 128.)
//
// Every wait on the MMA barrier is bounded; on expiry the kernel records
// kErrTimeout, stops taking items, frees its TMEM and returns.
#pragma once

#include "ra_common.cuh"
#include "ra_tilesg.cuh"

namespace ra {

constexpr int kTcRows = 128;     // rows per item (= kGenRows) = TMEM lanes
constexpr int kTcCols = 64;      // points per column tile (MMA N of GEMM 1)
constexpr int kTcThreads = 128;
constexpr unsigned kTcSpinLimit = 1u << 22;  // polls of the MMA barrier before giving up

__host__ __device__ constexpr int tc_tmem_cols(int DP) {
  return 3 * DP + 2 * kTcCols <= 256 ? 256 : 512;
}
__host__ __device__ constexpr size_t tc_smem_bytes(int DP) {
  // Y_hi, Y_lo, Yt_hi, Yt_lo, column weights, 8 partial |y'|^2 per point,
  // their totals and the totals less log2 b, barrier and TMEM address
  return (size_t)4 * kTcCols * DP * 4 + kTcCols * 4 * 11 + 16;
}
// Dynamic shared memory requested per CTA: enough that no more CTAs share an
// SM than its 512 TMEM columns hold (a CTA that cannot allocate would wait
// for a neighbour's whole persistent loop).
__host__ __device__ constexpr size_t tc_smem_request(int DP) {
  return tc_tmem_cols(DP) == 512 ? (tc_smem_bytes(DP) > (size_t)120 * 1024 ? tc_smem_bytes(DP)
                                                                           : (size_t)120 * 1024)
                                 : (size_t)80 * 1024;
}

// ---- tcgen05 / mbarrier primitives (PTX ISA 8.6+, sm_100a) -----------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
// Canonical no-swizzle shared-memory matrix descriptor (sm_100 version 1).
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}
// Instruction descriptor: D f32, A/B tf32, M = 128, N, B major (0 K, 1 MN).
__host__ __device__ constexpr uint32_t tc_idesc(int N, int b_major) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)b_major << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
}
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  const uint32_t zero = 0;  // disable-output-lane mask: every lane written
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(zero));
}
__device__ __forceinline__ void tc_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   mbar)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// true when the barrier completed phase `parity` within `limit` polls
__device__ __forceinline__ bool mbar_wait(uint32_t mbar, uint32_t parity,
                                          unsigned limit = kTcSpinLimit) {
  for (unsigned it = 0; it < limit; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred P1;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, P1;\n\t}\n"
        : "=r"(done)
        : "r"(mbar), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}
// 16 consecutive TMEM columns of this thread's lane <-> 16 registers
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
// 32 consecutive TMEM columns of this thread's lane <-> 32 registers
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

template <bool V>
struct BoolC {
  static constexpr bool value = V;
};

// a[u] for a runtime u in 0..3 by selects (no local-memory array)
__device__ __forceinline__ uint32_t sel4(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         int u) {
  const uint32_t lo = (u & 1) ? a1 : a0, hi = (u & 1) ? a3 : a2;
  return (u & 2) ? hi : lo;
}
// ---- the kernel -------------------------------------------------------------
template <int DP, int MODE>
__global__ void __launch_bounds__(kTcThreads, 1) tilestc_kernel(TilesGArgs A) {
  static_assert(DP == 32 || DP == 64 || DP == 128, "tensor-core path: DP in {32, 64, 128}");
  constexpr bool GRAD = MODE >= 1;
  constexpr bool SIG = MODE == 2;
  constexpr int NCOLS = tc_tmem_cols(DP);
  constexpr int C_XH = 0, C_XL = DP, C_S = 2 * DP, C_PL = 2 * DP + kTcCols,
                C_T = 2 * DP + 2 * kTcCols;
  constexpr int NCH = DP / 4;  // 16-byte chunks per point
  constexpr uint32_t IDESC1 = tc_idesc(kTcCols, 0), IDESC2 = tc_idesc(DP, 0);
  constexpr int NQ = kTcCols / 4;  // 4-point chunks of a column tile

  extern __shared__ __align__(1024) uint8_t tc_smem[];
  uint8_t *yhi = tc_smem;
  uint8_t *ylo = tc_smem + kTcCols * DP * 4;
  uint8_t *yth = tc_smem + 2 * kTcCols * DP * 4;
  uint8_t *ytl = tc_smem + 3 * kTcCols * DP * 4;
  float *bcol = reinterpret_cast<float *>(tc_smem + 4 * kTcCols * DP * 4);
  float *ysq = bcol + kTcCols;        // [8][64] partial |y'|^2
  float *ytot = ysq + 8 * kTcCols;    // [64] their totals, summed in order
  float *yqf = ytot + kTcCols;        // [64] |y'|^2 - log2 b (folded weight)
  uint64_t *mbar = reinterpret_cast<uint64_t *>(yqf + kTcCols);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mbar + 1);
  __shared__ double red[kTcThreads / 32 * 2];

  const int tid = threadIdx.x, warp = tid >> 5;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(NCOLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(mbar)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tlane = tbase + ((uint32_t)(warp * 32) << 16);  // this warp's lanes
  const uint32_t mb = smem_u32(mbar);
  uint32_t phase = 0;
  bool ok = true;
  bool pending = false;  // thread 0: a commit to `mb` not yet waited for

  const int64_t n_items = *A.n_items;
  for (int64_t it = (int64_t)blockIdx.x * A.shard_count + A.shard_index; it < n_items && ok;
       it += (int64_t)gridDim.x * A.shard_count) {
    const Item item = A.items[it];
    const Seg sg = A.seg[item.pair];
    const int o = item.block;  // 0: x-y, 1: x-x, 2: y-y, 3: y-x
    const bool rows_x = (o == 0 || o == 1), cols_x = (o == 1 || o == 3);
    const bool self = (o == 1 || o == 2);
    const int64_t rbase = rows_x ? sg.xs : sg.ys, rcnt = rows_x ? sg.xcount : sg.ycount;
    const int64_t cbase = cols_x ? sg.xs : sg.ys, ccnt = cols_x ? sg.xcount : sg.ycount;
    const float *Gr = rows_x ? A.Gx : A.Gy;
    const float *Ar = rows_x ? A.Ax : A.Ay;
    const float *Gc = cols_x ? A.Gx : A.Gy;
    const float *Ac = cols_x ? A.Ax : A.Ay;
    float *acc = rows_x ? A.accX : A.accY;
    const bool crossb = (o == 0 || o == 3);
    const int toff = crossb ? DP : 0, soff = 2 * DP + (crossb ? 1 : 0);
    const int64_t row = (int64_t)item.tile * kTcRows + tid;
    const bool rv = row < rcnt;
    const float a = rv ? Ar[rbase + row] : 0.f;

    // ---- this row -> X_hi / X_lo in TMEM (lane = row), |x'|^2 ----------------
    float xsq = 0.f;
    {
      // chunks of 32 coordinates, the next one loading while this one is
      // split and written to TMEM
      const float4 *src = reinterpret_cast<const float4 *>(Gr + (rbase + row) * DP);
      float4 cur[8], nxt[8];
#pragma unroll
      for (int q8 = 0; q8 < 8; ++q8) cur[q8] = rv ? src[q8] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
      for (int d0 = 0; d0 < DP; d0 += 32) {
        if (d0 + 32 < DP) {
#pragma unroll
          for (int q8 = 0; q8 < 8; ++q8)
            nxt[q8] = rv ? src[(d0 + 32) / 4 + q8] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        uint32_t h[32], l[32];
#pragma unroll
        for (int q8 = 0; q8 < 8; ++q8) {
          const float e[4] = {cur[q8].x, cur[q8].y, cur[q8].z, cur[q8].w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            xsq = fmaf(e[u], e[u], xsq);
            h[4 * q8 + u] = to_tf32(e[u]);
            l[4 * q8 + u] = to_tf32(e[u] - __uint_as_float(h[4 * q8 + u]));
          }
        }
        tmem_st32(tlane + C_XH + d0, h);
        tmem_st32(tlane + C_XL + d0, l);
#pragma unroll
        for (int q8 = 0; q8 < 8; ++q8) cur[q8] = nxt[q8];
      }
    }
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");

    // Column tiles are loaded into registers one tile ahead: thread t takes
    // 4-point x 4-coordinate blocks (point group q, coordinates 4c..4c+3 for
    // c = c0 + 8 i), all loads of a tile in flight at once; the next tile's
    // loads are issued right after GEMM 2 of this one is launched.  The
    // (q, c0) assignment makes every 8-thread phase of a 16-byte store hit 8
    // distinct bank groups in both layouts: q & 1 = t2, c0 & 1 = t0 ^ t2,
    // and the store order rotates with t & 3.
    constexpr int KB = NCH / (kTcThreads / NQ);  // blocks per thread
    static_assert(NQ == 16 && kTcThreads == 128, "thread mapping assumes 16 x 8");
    const int tb0 = tid & 1, tb1 = (tid >> 1) & 1, tb2 = (tid >> 2) & 1;
    const int q = tb2 | (tb1 << 1) | (((tid >> 3) & 3) << 2);
    const int c0 = (tb0 ^ tb2) | (((tid >> 5) & 3) << 1), rot = tid & 3;
    float4 E[KB][4];
    float bw[4];
    auto load_tile = [&](int64_t jt) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t j = jt + 4 * q + u;
        const bool cv = j < ccnt;
        const float4 *src = reinterpret_cast<const float4 *>(Gc + (cbase + j) * DP);
#pragma unroll
        for (int kb = 0; kb < KB; ++kb)
          E[kb][u] = cv ? src[c0 + kb * (kTcThreads / NQ)] : make_float4(0.f, 0.f, 0.f, 0.f);
        bw[u] = (c0 == 0 && cv) ? Ac[cbase + j] : 0.f;
      }
    };
    // Split into tf32 hi/lo and store both K-major layouts; the order of the
    // four 16-byte stores is rotated by lane so that a quarter-warp touches
    // at least four distinct bank groups.
    auto store_tile = [&](int64_t jt) {
      float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kb = 0; kb < KB; ++kb) {
        const int c = c0 + kb * (kTcThreads / NQ);
        uint32_t hh[4][4], ll[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float e[4] = {E[kb][u].x, E[kb][u].y, E[kb][u].z, E[kb][u].w};
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            part[u] = fmaf(e[v], e[v], part[u]);
            hh[u][v] = to_tf32(e[v]);
            ll[u][v] = to_tf32(e[v] - __uint_as_float(hh[u][v]));
          }
        }
#pragma unroll
        for (int s4 = 0; s4 < 4; ++s4) {
          const int u = (s4 + rot) & 3;  // point (row layout) / coordinate (transposed)
          const int jo = c * (kTcCols * 16) + (4 * q + u) * 16;
          uint32_t H[4], Lw[4], Ht[4], Lt[4];
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            H[v] = sel4(hh[0][v], hh[1][v], hh[2][v], hh[3][v], u);
            Lw[v] = sel4(ll[0][v], ll[1][v], ll[2][v], ll[3][v], u);
            Ht[v] = sel4(hh[v][0], hh[v][1], hh[v][2], hh[v][3], u);
            Lt[v] = sel4(ll[v][0], ll[v][1], ll[v][2], ll[v][3], u);
          }
          *reinterpret_cast<uint4 *>(yhi + jo) = make_uint4(H[0], H[1], H[2], H[3]);
          *reinterpret_cast<uint4 *>(ylo + jo) = make_uint4(Lw[0], Lw[1], Lw[2], Lw[3]);
          const int d = 4 * c + u;
          const int to = (d >> 3) * (NQ * 128) + q * 128 + (d & 7) * 16;
          *reinterpret_cast<uint4 *>(yth + to) = make_uint4(Ht[0], Ht[1], Ht[2], Ht[3]);
          *reinterpret_cast<uint4 *>(ytl + to) = make_uint4(Lt[0], Lt[1], Lt[2], Lt[3]);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) ysq[c0 * kTcCols + 4 * q + u] = part[u];
      if (c0 == 0) {
#pragma unroll
        for (int u = 0; u < 4; ++u) bcol[4 * q + u] = bw[u];
      }
      (void)jt;
    };
    if (ccnt > 0) load_tile(0);

    float s = 0.f, sig = 0.f;
    double s64 = 0.0, sg64 = 0.0;
    bool first = true;
    const float nxsq = -xsq;
    const int64_t row0 = (int64_t)item.tile * kTcRows;  // first row of the item
#pragma unroll 1
    for (int64_t j0 = 0; j0 < ccnt && ok; j0 += kTcCols) {
      // ---- column tile (registers, loaded earlier) -> Y in smem, |y'|^2 ------
      store_tile(j0);
      fence_async_smem();
      tc_fence_before();
      // a negative column weight cannot be folded into the exponent
      const bool anyneg = __syncthreads_or(c0 == 0 && (bw[0] < 0.f || bw[1] < 0.f ||
                                                       bw[2] < 0.f || bw[3] < 0.f)) != 0;
      tc_fence_after();

      // ---- GEMM 1: S = X Y^T (3xTF32), one thread issues -------------------
      if (tid == 0 && !A.no_mma) {
        const uint32_t sh = smem_u32(yhi), sl = smem_u32(ylo);
#pragma unroll
        for (int k = 0; k < DP / 8; ++k) {
          // K-major B: LBO = next 4 coordinates (1024 B), SBO = next 8 points (128 B)
          const uint64_t bh = tc_desc(sh + 2 * k * (kTcCols * 16), kTcCols * 16, 128);
          const uint64_t bl = tc_desc(sl + 2 * k * (kTcCols * 16), kTcCols * 16, 128);
          tc_mma(tbase + C_S, tbase + C_XH + 8 * k, bh, IDESC1, k > 0 ? 1u : 0u);
          tc_mma(tbase + C_S, tbase + C_XH + 8 * k, bl, IDESC1, 1u);
          tc_mma(tbase + C_S, tbase + C_XL + 8 * k, bh, IDESC1, 1u);
        }
        tc_commit(mb);
        pending = true;
      }
      // |y'|^2 totals for the epilogue, while GEMM 1 runs (published by the
      // barrier after its wait)
      if (tid < kTcCols) {
        float t = 0.f;
#pragma unroll
        for (int g = 0; g < kTcThreads / NQ; ++g) t += ysq[g * kTcCols + tid];
        ytot[tid] = t;
        yqf[tid] = t - log2f(bcol[tid]);  // +inf for zero weight and padding
      }
      // the decision to stop is taken by the whole CTA at once
      if (__syncthreads_or(!mbar_wait(mb, phase, A.spin_limit))) {
        ok = false;
        break;
      }
      pending = false;
      phase ^= 1u;
      tc_fence_after();

      // ---- epilogue of the tile: k, w, row sums, P = w (hi/lo) -> TMEM -------
      const int64_t dj = row - j0;  // this row's diagonal column in the tile
      const int diag = (self && dj >= 0 && dj < kTcCols) ? (int)dj : -1;
      float st = 0.f, sgt = 0.f;
      auto epilogue = [&](auto fold_t, auto diag_t) {
        constexpr bool FOLD = decltype(fold_t)::value, DG = decltype(diag_t)::value;
#pragma unroll 1
        for (int cb = 0; cb < kTcCols; cb += 32) {
          float S[32];
          tmem_ld32(tlane + C_S + cb, S);
          uint32_t ph[32], pl[32];
#pragma unroll
          for (int u = 0; u < 32; ++u) {
            const int j = cb + u;
            float w, r2 = 0.f;
            if (FOLD) {
              w = ex2(fmaf(2.f, S[u], nxsq - yqf[j]));  // b_j 2^(-r^2)
              if (SIG) r2 = fmaxf(xsq + ytot[j] - 2.f * S[u], 0.f);
            } else {
              r2 = fmaxf(xsq + ytot[j] - 2.f * S[u], 0.f);
              w = bcol[j] * ex2(-r2);
            }
            if (DG && j == diag) w = 0.f;
            st += w;
            if (SIG) sgt = fmaf(w, r2, sgt);
            const float hi = __uint_as_float(__float_as_uint(w) & 0xFFFFE000u);
            ph[u] = __float_as_uint(hi);
            pl[u] = __float_as_uint(w - hi);
          }
          if (GRAD) {
            tmem_st32(tlane + C_S + cb, ph);  // P_hi overwrites S (already read)
            tmem_st32(tlane + C_PL + cb, pl);
          }
        }
      };
      // the tile meets the diagonal of a self block (CTA-uniform)
      const bool dtile = self && j0 < row0 + kTcRows && row0 < j0 + kTcCols;
      if (anyneg)
        epilogue(BoolC<false>{}, BoolC<true>{});
      else if (dtile)
        epilogue(BoolC<true>{}, BoolC<true>{});
      else
        epilogue(BoolC<true>{}, BoolC<false>{});
      s += st;
      s64 += (double)st;
      if (SIG) {
        sig += sgt;
        sg64 += (double)sgt;
      }
      if (GRAD) {
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // ---- GEMM 2: T += P Y (3xTF32), B = the transposed Y tile -----------
        if (tid == 0 && !A.no_mma) {
          const uint32_t sh = smem_u32(yth), sl = smem_u32(ytl);
#pragma unroll
          for (int k = 0; k < kTcCols / 8; ++k) {
            // K-major B (N = d, K = j): LBO = next 4 points (128 B), SBO = next 8
            // coordinates (2048 B); a K step of 8 points is 2 chunks = 256 B
            const uint64_t bh = tc_desc(sh + k * 256, 128, NQ * 128);
            const uint64_t bl = tc_desc(sl + k * 256, 128, NQ * 128);
            tc_mma(tbase + C_T, tbase + C_S + 8 * k, bh, IDESC2, (first && k == 0) ? 0u : 1u);
            tc_mma(tbase + C_T, tbase + C_S + 8 * k, bl, IDESC2, 1u);
            tc_mma(tbase + C_T, tbase + C_PL + 8 * k, bh, IDESC2, 1u);
          }
          tc_commit(mb);
          pending = true;
        }
        if (j0 + kTcCols < ccnt) load_tile(j0 + kTcCols);  // in flight during GEMM 2
        if (__syncthreads_or(!mbar_wait(mb, phase, A.spin_limit))) {
          ok = false;
          break;
        }
        pending = false;
        phase ^= 1u;
        tc_fence_after();
        first = false;
      } else {
        // the next tile overwrites Y and S: every thread must be done with them
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (j0 + kTcCols < ccnt) load_tile(j0 + kTcCols);
      }
    }
    if (!ok) break;

    // ---- item outputs ---------------------------------------------------------
    if (GRAD && A.need_rows) {
      float *dst = acc + (rbase + row) * gen_acc_stride(DP);
#pragma unroll 1
      for (int d0 = 0; d0 < DP; d0 += 32) {
        float T[32];
        if (first) {
#pragma unroll
          for (int u = 0; u < 32; ++u) T[u] = 0.f;  // no column tile: T = 0
        } else {
          tmem_ld32(tlane + C_T + d0, T);
        }
        if (rv) {
#pragma unroll
          for (int u = 0; u < 32; u += 4)
            *reinterpret_cast<float4 *>(dst + toff + d0 + u) =
                make_float4(T[u], T[u + 1], T[u + 2], T[u + 3]);
        }
      }
      if (rv) dst[soff] = s;
    }
    (void)sig;
    // pair partials (x-y, x-x, y-y; y-x would count Kxy twice); a self block
    // adds the diagonal a_i^2 k_ii = a_i^2 left out of the row sums
    double kv = (double)a * (s64 + (self ? (double)a : 0.0)), sv = (double)a * sg64;
    kv = warp_sum(kv);
    sv = warp_sum(sv);
    if ((tid & 31) == 0) {
      red[warp] = kv;
      red[kTcThreads / 32 + warp] = sv;
    }
    tc_fence_before();
    __syncthreads();  // also: every thread is done reading T before the next item
    tc_fence_after();
    if (tid == 0) {
      double K = 0.0, Sg = 0.0;
      for (int w = 0; w < kTcThreads / 32; ++w) {
        K += red[w];
        Sg += red[kTcThreads / 32 + w];
      }
      A.itemK[it] = o == 3 ? 0.0 : K;
      A.itemS[it] = o == 3 ? 0.0 : Sg;
    }
    __syncthreads();  // `red` is rewritten by the next item, possibly without a column tile
  }
  if (!ok && tid == 0) {
    atomicOr(A.err, (int)kErrTimeout);
    // give the MMAs in flight a last bounded chance to land before TMEM is
    // freed (the full limit, whatever the waits above used)
    if (pending) (void)mbar_wait(mb, phase);
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
