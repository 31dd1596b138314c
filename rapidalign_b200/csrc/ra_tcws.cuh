// ra_tcws.cuh -- warp-specialised tensor-core kernel of the generic layout
// for padded dimensions DP in {64, 128} (one CTA per SM: all 512 TMEM
// columns).  Same items, TMEM and shared-memory operand layouts, arithmetic
// and outputs as tilestc_kernel (ra_tc.cuh); what changes is who does what:
//
//   warps 0-3  epilogue: thread t = row t = TMEM lane t.  Per item: the row
//              tile into TMEM (X hi/lo), then per column tile: S from TMEM,
//              w = b 2^(-r^2), row sums, P = w (hi/lo) back into TMEM; at the
//              end of the item T from TMEM and the per-point records.
//   warps 4-7  producers: per column tile, the global loads, the tf32 hi/lo
//              split and the stores of the two shared-memory operand layouts
//              (Y for GEMM 1 once GEMM 1 of the previous tile is done, its
//              transpose for GEMM 2 once GEMM 2 of the previous tile is done),
//              the |y'|^2 totals and the weights.
//   warp 8     lane 0 issues the MMAs: GEMM 1 of tile j as soon as its Y is
//              stored and GEMM 2 of tile j-1 is done, GEMM 2 of tile j as
//              soon as P and the transposed Y are ready.
// So while the epilogue works on tile j, the producers store tile j+1, and
// the tensor core runs GEMM 2 of tile j and GEMM 1 of tile j+1 back to back.
//
// Hand-offs are mbarriers, one completion per column tile (x_full: per
// item).  Each role waits on every completion it needs in order, and no
// role can complete a barrier twice before its waiters have seen the first
// completion (the producers hold the Y-ready signal of tile j+1 until the
// epilogue has handed over tile j), so a parity bit per wait is exact.
// Every wait is bounded and also gives up when another role has aborted.
// The epilogue and producer roles turn each wait's outcome into one
// decision for the whole role (a barrier-reduction) before they go on, so a
// role never leaves its loop with some threads still inside it.  On expiry
// the kernel records kErrTimeout, drains the MMAs it issued (bounded), frees
// its TMEM and returns.
#pragma once

#include "ra_tc.cuh"

namespace ra {

constexpr int kWsEpiWarps = 4;
constexpr int kWsProdWarps = 4;
constexpr int kWsMmaWarp = kWsEpiWarps + kWsProdWarps;  // warp 8
constexpr int kWsThreads = 32 * (kWsMmaWarp + 1);       // 288

// Shared memory after the four operand tiles: bcol / ytot / yqf per tile
// parity, 8 partial |y'|^2 rows, flags, 6 mbarriers, the TMEM address and
// the epilogue's reduction slots.
constexpr int kWsSmallFloats = 6 * kTcCols + 8 * kTcCols;
__host__ __device__ constexpr size_t tc_ws_smem_bytes(int DP) {
  return (size_t)4 * kTcCols * DP * 4 + kWsSmallFloats * 4 + 16 + 6 * 8 + 8 + 8 * 8;
}
__host__ __device__ constexpr size_t tc_ws_smem_request(int DP) {
  // at least 120 KB: never two CTAs on one SM (each takes all 512 columns)
  return tc_ws_smem_bytes(DP) > (size_t)120 * 1024 ? tc_ws_smem_bytes(DP) : (size_t)120 * 1024;
}

__device__ __forceinline__ void mbar_init(uint32_t a, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t a) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}
// Wait for the phase of the given parity; false when `limit` polls are
// reached or another role has raised the abort flag.
__device__ __forceinline__ bool ws_wait(uint32_t mbar, uint32_t parity,
                                        const volatile int *abort_flag, unsigned limit) {
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
    if ((it & 31) == 31 && *abort_flag) return false;
  }
  return false;
}
// Named barrier among the threads of one role (ids 1 and 2; 0 is
// __syncthreads).
__device__ __forceinline__ void role_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ int role_sync_or(int id, int nthreads, int pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.s32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.s32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(pred), "r"(id), "r"(nthreads)
      : "memory");
  return r;
}

template <int DP, int MODE>
__global__ void __launch_bounds__(kWsThreads, 1) tilestc_ws_kernel(TilesGArgs A) {
  static_assert(DP == 64 || DP == 128, "warp-specialised path: DP in {64, 128}");
  constexpr bool GRAD = MODE >= 1;
  constexpr bool SIG = MODE == 2;
  constexpr int NCOLS = 512;
  static_assert(tc_tmem_cols(DP) == NCOLS, "one CTA per SM");
  constexpr int C_XH = 0, C_XL = DP, C_S = 2 * DP, C_PL = 2 * DP + kTcCols,
                C_T = 2 * DP + 2 * kTcCols;
  constexpr int NCH = DP / 4;
  constexpr uint32_t IDESC1 = tc_idesc(kTcCols, 0), IDESC2 = tc_idesc(DP, 0);
  constexpr int NQ = kTcCols / 4;
  constexpr int PT = 32 * kWsProdWarps;  // producer threads
  constexpr int ET = 32 * kWsEpiWarps;   // epilogue threads

  extern __shared__ __align__(1024) uint8_t ws_smem[];
  uint8_t *yhi = ws_smem;
  uint8_t *ylo = ws_smem + kTcCols * DP * 4;
  uint8_t *yth = ws_smem + 2 * kTcCols * DP * 4;
  uint8_t *ytl = ws_smem + 3 * kTcCols * DP * 4;
  float *small = reinterpret_cast<float *>(ws_smem + 4 * kTcCols * DP * 4);
  float *bcol = small;                 // [2][64] column weights
  float *ytot = small + 2 * kTcCols;   // [2][64] |y'|^2
  float *yqf = small + 4 * kTcCols;    // [2][64] |y'|^2 - log2 b
  float *ysq = small + 6 * kTcCols;    // [8][64] partial |y'|^2 (producers only)
  int *negf = reinterpret_cast<int *>(small + kWsSmallFloats);  // [2] tile has b < 0
  volatile int *abortf = negf + 2;
  uint64_t *bars = reinterpret_cast<uint64_t *>(negf + 4);  // 8-byte aligned
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 6);
  double *red = reinterpret_cast<double *>(tmem_slot + 2);  // [8]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t b_xfull = smem_u32(bars + 0), b_ykfull = smem_u32(bars + 1),
                 b_ytfull = smem_u32(bars + 2), b_g1 = smem_u32(bars + 3),
                 b_pfull = smem_u32(bars + 4), b_g2 = smem_u32(bars + 5);
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(NCOLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    mbar_init(b_xfull, ET);
    mbar_init(b_ykfull, PT);
    mbar_init(b_ytfull, PT);
    mbar_init(b_g1, 1);
    mbar_init(b_pfull, ET);
    mbar_init(b_g2, 1);
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

  if (warp < kWsEpiWarps) {
    // =================== epilogue warps: rows, S -> P, T ===================
    const uint32_t tlane = tbase + ((uint32_t)(warp * 32) << 16);
    uint32_t t = 0;  // column tiles seen (all items)
    for (int64_t it = ifirst; it < n_items; it += istep) {
      const Item item = A.items[it];
      const Seg sg = A.seg[item.pair];
      const int o = item.block;  // 0: x-y, 1: x-x, 2: y-y, 3: y-x
      const bool rows_x = (o == 0 || o == 1), cols_x = (o == 1 || o == 3);
      const bool self = (o == 1 || o == 2);
      const int64_t rbase = rows_x ? sg.xs : sg.ys, rcnt = rows_x ? sg.xcount : sg.ycount;
      const int64_t ccnt = cols_x ? sg.xcount : sg.ycount;
      const float *Gr = rows_x ? A.Gx : A.Gy;
      const float *Ar = rows_x ? A.Ax : A.Ay;
      float *acc = rows_x ? A.accX : A.accY;
      const bool crossb = (o == 0 || o == 3);
      const int toff = crossb ? DP : 0, soff = 2 * DP + (crossb ? 1 : 0);
      const int64_t row0 = (int64_t)item.tile * kTcRows;
      const int64_t row = row0 + tid;
      const bool rv = row < rcnt;
      const float a = rv ? Ar[rbase + row] : 0.f;
      const int ntiles = (int)ceil_div(ccnt, (int64_t)kTcCols);
      float s = 0.f, sig = 0.f;
      double s64 = 0.0, sg64 = 0.0;
      float xsq = 0.f;
      bool ok = true;
      if (ntiles > 0) {
        // ---- this row -> X_hi / X_lo in TMEM (lane = row), |x'|^2 ----------
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
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        mbar_arrive(b_xfull);
        const float nxsq = -xsq;

        for (int jt = 0; jt < ntiles; ++jt, ++t) {
          const int64_t j0 = (int64_t)jt * kTcCols;
          // the tile's weights and totals (producers), then S (GEMM 1)
          const bool w_ok = ws_wait(b_ykfull, t & 1u, abortf, A.spin_limit) &&
                            ws_wait(b_g1, t & 1u, abortf, A.spin_limit);
          if (role_sync_or(1, ET, !w_ok)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int pb = (int)(t & 1u);
          const float *bc = bcol + pb * kTcCols, *yt = ytot + pb * kTcCols,
                      *yq = yqf + pb * kTcCols;
          const bool anyneg = negf[pb] != 0;
          const int64_t dj = row - j0;
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
                  w = ex2(fmaf(2.f, S[u], nxsq - yq[j]));  // b_j 2^(-r^2)
                  if (SIG) r2 = fmaxf(xsq + yt[j] - 2.f * S[u], 0.f);
                } else {
                  r2 = fmaxf(xsq + yt[j] - 2.f * S[u], 0.f);
                  w = bc[j] * ex2(-r2);
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
          if (GRAD) asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          tc_fence_before();
          mbar_arrive(b_pfull);  // P ready (and S consumed)
        }
        if (ok && GRAD) {
          // T of the item: after GEMM 2 of its last tile
          const bool w_ok = ws_wait(b_g2, (t - 1u) & 1u, abortf, A.spin_limit);
          if (role_sync_or(1, ET, !w_ok)) ok = false;
          tc_fence_after();
        }
      }
      if (!ok) {
        fail();
        break;
      }

      // ---- item outputs -----------------------------------------------------
      if (GRAD && A.need_rows) {
        float *dst = acc + (rbase + row) * gen_acc_stride(DP);
#pragma unroll 1
        for (int d0 = 0; d0 < DP; d0 += 32) {
          float T[32];
          if (ntiles == 0) {
#pragma unroll
            for (int u = 0; u < 32; ++u) T[u] = 0.f;
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
      double kv = (double)a * (s64 + (self ? (double)a : 0.0)), sv = (double)a * sg64;
      kv = warp_sum(kv);
      sv = warp_sum(sv);
      if (lane == 0) {
        red[warp] = kv;
        red[kWsEpiWarps + warp] = sv;
      }
      role_sync(1, ET);
      if (tid == 0) {
        double K = 0.0, Sg = 0.0;
        for (int w = 0; w < kWsEpiWarps; ++w) {
          K += red[w];
          Sg += red[kWsEpiWarps + w];
        }
        A.itemK[it] = o == 3 ? 0.0 : K;
        A.itemS[it] = o == 3 ? 0.0 : Sg;
      }
      role_sync(1, ET);  // `red` is rewritten by the next item
    }
  } else if (warp < kWsMmaWarp) {
    // =================== producer warps: Y tiles into shared memory =========
    const int ptid = tid - ET;
    constexpr int KB = NCH / (PT / NQ);
    static_assert(NQ == 16 && PT == 128, "thread mapping assumes 16 x 8");
    const int tb0 = ptid & 1, tb1 = (ptid >> 1) & 1, tb2 = (ptid >> 2) & 1;
    const int q = tb2 | (tb1 << 1) | (((ptid >> 3) & 3) << 2);
    const int c0 = (tb0 ^ tb2) | (((ptid >> 5) & 3) << 1), rot = ptid & 3;
    uint32_t t = 0;
    for (int64_t it = ifirst; it < n_items; it += istep) {
      const Item item = A.items[it];
      const Seg sg = A.seg[item.pair];
      const int o = item.block;
      const bool cols_x = (o == 1 || o == 3);
      const int64_t cbase = cols_x ? sg.xs : sg.ys, ccnt = cols_x ? sg.xcount : sg.ycount;
      const float *Gc = cols_x ? A.Gx : A.Gy;
      const float *Ac = cols_x ? A.Ax : A.Ay;
      const int ntiles = (int)ceil_div(ccnt, (int64_t)kTcCols);
      bool ok = true;
      for (int jt = 0; jt < ntiles; ++jt, ++t) {
        const int64_t j0 = (int64_t)jt * kTcCols;
        const int pb = (int)(t & 1u);
        // loads first: they need no buffer
        float4 E[KB][4];
        float bw[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t j = j0 + 4 * q + u;
          const bool cv = j < ccnt;
          const float4 *src = reinterpret_cast<const float4 *>(Gc + (cbase + j) * DP);
#pragma unroll
          for (int kb = 0; kb < KB; ++kb)
            E[kb][u] = cv ? src[c0 + kb * (PT / NQ)] : make_float4(0.f, 0.f, 0.f, 0.f);
          bw[u] = (c0 == 0 && cv) ? Ac[cbase + j] : 0.f;
        }
        // Y (GEMM 1 layout) is free once GEMM 1 of the previous tile is done;
        // the barrier also orders the previous tile's reads of ysq
        const bool w1 = t == 0 || ws_wait(b_g1, (t - 1u) & 1u, abortf, A.spin_limit);
        if (role_sync_or(2, PT, !w1)) {
          ok = false;
          break;
        }
        float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kb = 0; kb < KB; ++kb) {
          const int c = c0 + kb * (PT / NQ);
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
            const int u = (s4 + rot) & 3;
            const int jo = c * (kTcCols * 16) + (4 * q + u) * 16;
            uint32_t H[4], Lw[4];
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              H[v] = sel4(hh[0][v], hh[1][v], hh[2][v], hh[3][v], u);
              Lw[v] = sel4(ll[0][v], ll[1][v], ll[2][v], ll[3][v], u);
            }
            *reinterpret_cast<uint4 *>(yhi + jo) = make_uint4(H[0], H[1], H[2], H[3]);
            *reinterpret_cast<uint4 *>(ylo + jo) = make_uint4(Lw[0], Lw[1], Lw[2], Lw[3]);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) ysq[c0 * kTcCols + 4 * q + u] = part[u];
        if (c0 == 0) {
#pragma unroll
          for (int u = 0; u < 4; ++u) bcol[pb * kTcCols + 4 * q + u] = bw[u];
        }
        const int negl = c0 == 0 && (bw[0] < 0.f || bw[1] < 0.f || bw[2] < 0.f || bw[3] < 0.f);
        fence_async_smem();
        const int anyneg = role_sync_or(2, PT, negl);
        if (ptid < kTcCols) {
          float tt = 0.f;
#pragma unroll
          for (int g = 0; g < PT / NQ; ++g) tt += ysq[g * kTcCols + ptid];
          ytot[pb * kTcCols + ptid] = tt;
          yqf[pb * kTcCols + ptid] = tt - log2f(bcol[pb * kTcCols + ptid]);
        }
        if (ptid == 0) negf[pb] = anyneg;
        // hand the tile over only after the epilogue took the previous one
        const bool w2 = t == 0 || ws_wait(b_pfull, (t - 1u) & 1u, abortf, A.spin_limit);
        if (role_sync_or(2, PT, !w2)) {
          ok = false;
          break;
        }
        mbar_arrive(b_ykfull);
        if (GRAD) {
          // transposed Y (GEMM 2) once GEMM 2 of the previous tile is done
          const bool w3 = t == 0 || ws_wait(b_g2, (t - 1u) & 1u, abortf, A.spin_limit);
          if (role_sync_or(2, PT, !w3)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int kb = 0; kb < KB; ++kb) {
            const int c = c0 + kb * (PT / NQ);
            uint32_t hh[4][4], ll[4][4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float e[4] = {E[kb][u].x, E[kb][u].y, E[kb][u].z, E[kb][u].w};
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                hh[u][v] = to_tf32(e[v]);
                ll[u][v] = to_tf32(e[v] - __uint_as_float(hh[u][v]));
              }
            }
#pragma unroll
            for (int s4 = 0; s4 < 4; ++s4) {
              const int u = (s4 + rot) & 3;
              const int d = 4 * c + u;
              const int to = (d >> 3) * (NQ * 128) + q * 128 + (d & 7) * 16;
              uint32_t H[4], Lw[4];
#pragma unroll
              for (int p = 0; p < 4; ++p) {
                H[p] = sel4(hh[p][0], hh[p][1], hh[p][2], hh[p][3], u);
                Lw[p] = sel4(ll[p][0], ll[p][1], ll[p][2], ll[p][3], u);
              }
              *reinterpret_cast<uint4 *>(yth + to) = make_uint4(H[0], H[1], H[2], H[3]);
              *reinterpret_cast<uint4 *>(ytl + to) = make_uint4(Lw[0], Lw[1], Lw[2], Lw[3]);
            }
          }
          fence_async_smem();
          mbar_arrive(b_ytfull);
        }
      }
      if (!ok) {
        fail();
        break;
      }
    }
  } else if (lane == 0) {
    // =================== MMA issuer =========================================
    uint32_t t = 0, xk = 0, n_g1 = 0, n_g2 = 0;  // tiles, items, commits issued
    bool ok = true;
    // (test hook: no MMA at all, so every wait on a GEMM expires)
    for (int64_t it = ifirst; it < n_items && ok && !*abortf && !A.no_mma; it += istep) {
      const Item item = A.items[it];
      const Seg sg = A.seg[item.pair];
      const bool cols_x = (item.block == 1 || item.block == 3);
      const int64_t ccnt = cols_x ? sg.xcount : sg.ycount;
      const int ntiles = (int)ceil_div(ccnt, (int64_t)kTcCols);
      if (ntiles == 0) continue;
      if (!ws_wait(b_xfull, xk & 1u, abortf, A.spin_limit)) {
        ok = false;
        break;
      }
      ++xk;
      for (int jt = 0; jt < ntiles; ++jt, ++t) {
        // GEMM 1 needs this tile's Y and a free S (GEMM 2, or without a
        // backward the epilogue, of the previous tile done)
        if (!ws_wait(b_ykfull, t & 1u, abortf, A.spin_limit) ||
            (t > 0 && !ws_wait(GRAD ? b_g2 : b_pfull, (t - 1u) & 1u, abortf, A.spin_limit))) {
          ok = false;
          break;
        }
        tc_fence_after();
        {
          const uint32_t sh = smem_u32(yhi), sl = smem_u32(ylo);
#pragma unroll
          for (int k = 0; k < DP / 8; ++k) {
            const uint64_t bh = tc_desc(sh + 2 * k * (kTcCols * 16), kTcCols * 16, 128);
            const uint64_t bl = tc_desc(sl + 2 * k * (kTcCols * 16), kTcCols * 16, 128);
            tc_mma(tbase + C_S, tbase + C_XH + 8 * k, bh, IDESC1, k > 0 ? 1u : 0u);
            tc_mma(tbase + C_S, tbase + C_XH + 8 * k, bl, IDESC1, 1u);
            tc_mma(tbase + C_S, tbase + C_XL + 8 * k, bh, IDESC1, 1u);
          }
          tc_commit(b_g1);
          ++n_g1;
        }
        if (GRAD) {
          if (!ws_wait(b_pfull, t & 1u, abortf, A.spin_limit) ||
              !ws_wait(b_ytfull, t & 1u, abortf, A.spin_limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sh = smem_u32(yth), sl = smem_u32(ytl);
#pragma unroll
          for (int k = 0; k < kTcCols / 8; ++k) {
            const uint64_t bh = tc_desc(sh + k * 256, 128, NQ * 128);
            const uint64_t bl = tc_desc(sl + k * 256, 128, NQ * 128);
            tc_mma(tbase + C_T, tbase + C_S + 8 * k, bh, IDESC2, (jt == 0 && k == 0) ? 0u : 1u);
            tc_mma(tbase + C_T, tbase + C_S + 8 * k, bl, IDESC2, 1u);
            tc_mma(tbase + C_T, tbase + C_PL + 8 * k, bh, IDESC2, 1u);
          }
          tc_commit(b_g2);
          ++n_g2;
        }
      }
    }
    if (!ok) fail();
    // every MMA issued has landed before TMEM is freed (bounded, also when
    // another role aborted; at most one GEMM of each kind is in flight)
    if (n_g1 > 0) (void)mbar_wait(b_g1, (n_g1 - 1u) & 1u);
    if (n_g2 > 0) (void)mbar_wait(b_g2, (n_g2 - 1u) & 1u);
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
