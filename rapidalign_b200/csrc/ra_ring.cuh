// ra_ring.cuh -- the wide-point (D >= 32) O(N) passes fed by bulk copies.
//
// A pass over the chunk map (ra_chunks.cuh) reads, for every point of a
// chunk, rows of fixed size that lie back to back in memory across the points
// of a segment: the caller's coordinates (D floats), the per-point sums of
// the tile kernel (gen_acc_stride(DP) floats), the normalised weights.  Here
// one producer lane takes the chunk tickets and streams each chunk's rows, a
// stage of R points at a time, into a ring of shared-memory stages with
// cp.async.bulk; eight consumer warps work from shared memory.  Every stage
// carries a header naming its chunk and rows, so the producer keeps copying
// across chunk boundaries while the consumers close a chunk: the loads in
// flight per CTA are the ring's bytes (tens of KB), not what registers hold,
// and no chunk start waits for a round trip to memory.
//
// Waits are bounded (kTcSpinLimit polls).  A role whose wait gives up raises
// the CTA's abort flag and records kErrTimeout; the others see the flag in
// their own waits and stop; the producer finally waits (bounded) for the
// copies it issued, so none lands after the CTA is gone.  The consumers'
// barriers are mbarriers (bounded, abortable), never bar.sync.
#pragma once

#include "ra_chunks.cuh"
#include "ra_epilogue.cuh"
#include "ra_prep.cuh"
#include "ra_tcprim.cuh"

namespace ra {

constexpr int kRingWarps = 8;                 // consumer warps
constexpr int kRingCons = 32 * kRingWarps;    // consumer threads
constexpr int kRingThreads = kRingCons + 32;  // + one producer warp
constexpr int kRingProdWarp = kRingWarps;
constexpr int kRingFirst = 1, kRingLast = 2, kRingStop = 4;  // RingHdr::flags

// What a stage holds: rows [r0, r0 + nr) of one chunk.
struct RingHdr {
  int64_t p, c, v, first, n;  // the chunk, as for_each_chunk names it
  int64_t s, r0, count;       // the side's first point and valid points; first row
  int64_t tb;                 // packing: the side's first tile
  double k_x, cs, cc;         // the side's constants (epi_side; packing: 1 / W, the
                              // fp16 coordinate and weight scales)
  float scl;                  // the pair's coordinate scale
  int side, nr, flags, aoff;  // aoff: byte offset of the stage's first weight
};

// How a ring kernel runs: the polls of one role wait (kTcSpinLimit), and, for
// tests of the failure path only, an idle producer that copies nothing, so
// the consumers' first wait expires with no copy in flight.  The producer's
// final drain keeps kTcSpinLimit whatever `limit` says.
struct RingRun {
  unsigned limit;
  int idle;
};

// The ring's shared state (static shared memory of the kernel).
template <int NS>
struct RingCtl {
  uint64_t full[NS], empty[NS];
  uint64_t cons;  // the consumers' barrier (kRingCons arrivals per phase)
  RingHdr hdr[NS];
  int abort;
};

template <int NS>
__device__ __forceinline__ void ring_init(RingCtl<NS> &R) {
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      mbar_init(smem_u32(&R.full[s]), 1);
      mbar_init(smem_u32(&R.empty[s]), kRingWarps);
    }
    mbar_init(smem_u32(&R.cons), kRingCons);
    R.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
}

// The chunk behind ticket v (the fields for_each_chunk passes).
__device__ __forceinline__ void ring_chunk(const ChunkMap &M, int64_t v, RingHdr &h) {
  const int64_t p = M.cpair[v];
  const int64_t lo = M.choff[p], hi = M.choff[p + 1];
  int64_t cx = M.chx[p];
  if (cx > hi - lo) cx = hi - lo;
  const int64_t local = v - lo;
  h.side = local < cx ? 0 : 1;
  h.c = h.side == 0 ? local : local - cx;
  h.first = h.side == 0 ? lo : lo + cx;
  h.n = h.side == 0 ? cx : (hi - lo) - cx;
  h.p = p;
  h.v = v;
}

// Producer lane.  rows(h, b, e) sets h.s and the chunk's row range [b, e);
// copy(h, dst, bar) adds the stage's bytes to `bar`'s expected transactions
// (mbar_tx, no arrival) and issues its bulk copies into shared address dst.
// The lane then stores the stage's header and arrives, the barrier's one
// arrival: the phase completes after both that and the copies.  Ends with a
// stop stage.  Returns the number of stages armed (for the drain).
template <int NS, typename Rows, typename Copy>
__device__ uint32_t ring_produce(const ChunkMap &M, RingCtl<NS> &R, uint32_t buf, uint32_t SB,
                                 int rows_per_stage, Rows rows, Copy copy, int *err,
                                 unsigned limit) {
  const int64_t total = M.choff[M.P];
  uint32_t k = 0;
  bool ok = true;
  // a free stage for stage number k (its previous use released by all warps)
  auto acquire = [&](int &s) {
    s = (int)(k % NS);
    if (k >= (uint32_t)NS &&
        !ws_wait(smem_u32(&R.empty[s]), ((k / NS) - 1) & 1, &R.abort, limit)) {
      if (!R.abort) atomicOr(err, (int)kErrTimeout);
      R.abort = 1;
      return false;
    }
    return true;
  };
  unsigned v = atomicAdd(M.ticket, 1u);
  while (ok && (int64_t)v < total) {
    const unsigned vn = atomicAdd(M.ticket, 1u);  // the next chunk, taken early
    RingHdr h;
    ring_chunk(M, v, h);
    int64_t b, e;
    rows(h, b, e);
    for (int64_t r0 = b; r0 < e; r0 += rows_per_stage) {
      int s;
      if (!acquire(s)) {
        ok = false;
        break;
      }
      h.r0 = r0;
      h.nr = (int)(e - r0 < rows_per_stage ? e - r0 : rows_per_stage);
      h.flags = (r0 == b ? kRingFirst : 0) | (r0 + rows_per_stage >= e ? kRingLast : 0);
      h.aoff = 0;
      copy(h, buf + (uint32_t)s * SB, smem_u32(&R.full[s]));  // may set h.aoff
      R.hdr[s] = h;  // visible to the consumers through the arrival (release)
      ++k;
      mbar_arrive(smem_u32(&R.full[s]));
    }
    v = vn;
  }
  if (ok) {
    int s;
    if (acquire(s)) {
      R.hdr[s].flags = kRingStop;
      ++k;
      mbar_arrive(smem_u32(&R.full[s]));
    }
  }
  return k;
}

// The producer's last act: every stage it armed has landed (bounded waits,
// whatever the abort flag says).
template <int NS>
__device__ void ring_drain(RingCtl<NS> &R, uint32_t k, unsigned limit) {
  const uint32_t j0 = k > (uint32_t)NS ? k - NS : 0;
  for (uint32_t j = j0; j < k; ++j) mbar_wait(smem_u32(&R.full[j % NS]), (j / NS) & 1, limit);
}

// Consumer warps: on_stage(h, stage pointer) for every stage until the stop
// stage; false when a wait gave up (or on_stage returned false).
template <int NS, typename OnStage>
__device__ bool ring_consume(RingCtl<NS> &R, const uint8_t *buf, uint32_t SB, OnStage on_stage,
                             int *err, unsigned limit) {
  const int lane = threadIdx.x & 31;
  for (uint32_t k = 0;; ++k) {
    const int s = (int)(k % NS);
    if (!ws_wait(smem_u32(&R.full[s]), (k / NS) & 1, &R.abort, limit)) {
      if (!R.abort) atomicOr(err, (int)kErrTimeout);
      R.abort = 1;
      return false;
    }
    const RingHdr h = R.hdr[s];
    if (h.flags & kRingStop) return true;
    if (!on_stage(h, buf + (size_t)s * SB)) return false;
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&R.empty[s]));
  }
}

// Barrier of the consumer threads (bounded, abortable).  `phase` counts the
// barriers this thread passed.
template <int NS>
__device__ __forceinline__ bool ring_cons_sync(RingCtl<NS> &R, uint32_t &phase, int *err,
                                               unsigned limit) {
  mbar_arrive(smem_u32(&R.cons));
  const bool ok = ws_wait(smem_u32(&R.cons), phase & 1, &R.abort, limit);
  ++phase;
  if (!ok) {
    if (!R.abort) atomicOr(err, (int)kErrTimeout);
    R.abort = 1;
  }
  return ok;
}

// ---------------------------------------------------------------------------
// Pass 1 (sums) for wide points with equal weights and no mask: the rows are
// the caller's coordinates.  Per chunk the same records as statsw4_kernel:
// rec[0] W, rec[1] valid count, rec[2] last valid row, rec[3 + d] sum w' p,
// rec[3 + DP + d] sum p, then the largest and smallest weight and the largest
// |coordinate|.  Lanes map to coordinates as in statsw4_kernel (LPP lanes per
// point, PPW points per warp step); the partials of the 8 warps are combined
// in warp order.
// ---------------------------------------------------------------------------
constexpr int kRingSumStages = 5;
constexpr uint32_t kRingSumStageBytes = 16384;

template <int DP>
__global__ void __launch_bounds__(kRingThreads, 2) statsw_ring_kernel(PrepArgs A,
                                                                       RingRun run) {
  const unsigned limit = run.limit;
  constexpr int NS = kRingSumStages, NW = kRingWarps, NC = DP / 4;
  constexpr int LPP = NC < 32 ? NC : 32;  // lanes per point
  constexpr int CPL = NC / LPP;           // float4 chunks per lane
  constexpr int PPW = 32 / LPP;           // points per warp step
  constexpr uint32_t SB = kRingSumStageBytes;
  extern __shared__ __align__(128) uint8_t ring_buf[];
  __shared__ RingCtl<NS> R;
  __shared__ double sh[NW][2 * DP + 2];
  __shared__ long long shl[NW];
  __shared__ float shm[NW][3];
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int D = A.D;
  const int rows = (int)(SB / (uint32_t)(D * 4));  // points per stage
  ring_init(R);

  if (wid == kRingProdWarp) {
    if (lane == 0 && !run.idle) {
      const uint32_t k = ring_produce(
          M, R, smem_u32(ring_buf), SB, rows,
          [&](RingHdr &h, int64_t &b, int64_t &e) {
            const Seg sg = A.seg[h.p];
            h.s = h.side == 0 ? sg.xs : sg.ys;
            const int64_t span = h.side == 0 ? sg.xspan : sg.yspan;
            b = h.c * kChunk;
            e = b + kChunk < span ? b + kChunk : span;
          },
          [&](RingHdr &h, uint32_t dst, uint32_t bar) {
            const float *pts = h.side == 0 ? A.x : A.y;
            const uint32_t bytes = (uint32_t)h.nr * (uint32_t)(D * 4);
            mbar_tx(bar, bytes);
            bulk_g2s(dst, pts + (h.s + h.r0) * D, bytes, bar);
          },
          A.err, limit);
      ring_drain(R, k, kTcSpinLimit);
    }
    return;
  }

  // ---- consumers ----
  const int cl = lane % LPP, q = lane / LPP;
  double acc[CPL][4], acc2[CPL][4], W = 0.0;  // two sets: even and odd warp steps
  long long last = -1;
  float cmax = 0.f;
  bool any = false;
  uint32_t phase = 0;
  ring_consume(
      R, ring_buf, SB,
      [&](const RingHdr &h, const uint8_t *st) -> bool {
        if (h.flags & kRingFirst) {
#pragma unroll
          for (int k = 0; k < CPL; ++k)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[k][j] = acc2[k][j] = 0.0;
          W = 0.0;
          last = -1;
          cmax = 0.f;
          any = false;
        }
        const float *sp = reinterpret_cast<const float *>(st);
        // every point weighs 1 and is valid (equal weights, no mask), so the
        // weighted and the plain coordinate sums are the same; two warp steps
        // per iteration into two accumulator sets (independent add chains)
        constexpr int STEP = NW * PPW;
        for (int r = wid * PPW + q; r < h.nr; r += 2 * STEP) {
          const int r2 = r + STEP;
          const bool two = r2 < h.nr;
#pragma unroll
          for (int k = 0; k < CPL; ++k) {
            const int cc = cl + LPP * k;
            if (4 * cc < D) {
              const float4 xv = *reinterpret_cast<const float4 *>(sp + (size_t)r * D + 4 * cc);
              const float4 xw = two ? *reinterpret_cast<const float4 *>(sp + (size_t)r2 * D + 4 * cc)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
              acc[k][0] += (double)xv.x;
              acc[k][1] += (double)xv.y;
              acc[k][2] += (double)xv.z;
              acc[k][3] += (double)xv.w;
              acc2[k][0] += (double)xw.x;
              acc2[k][1] += (double)xw.y;
              acc2[k][2] += (double)xw.z;
              acc2[k][3] += (double)xw.w;
              const float m0 = fmaxf(fmaxf(fabsf(xv.x), fabsf(xv.y)), fmaxf(fabsf(xv.z), fabsf(xv.w)));
              const float m1 = fmaxf(fmaxf(fabsf(xw.x), fabsf(xw.y)), fmaxf(fabsf(xw.z), fabsf(xw.w)));
              cmax = fmaxf(cmax, fmaxf(m0, m1));
            }
          }
          if (cl == 0) {
            W += two ? 2.0 : 1.0;
            last = h.r0 + (two ? r2 : r);
          }
          any = true;
        }
        if (!(h.flags & kRingLast)) return true;
        // ---- the chunk's records: warp slots, then the 8 warps in order ----
#pragma unroll
        for (int k = 0; k < CPL; ++k)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[k][j] += acc2[k][j];
#pragma unroll
        for (int o = LPP; o < 32; o <<= 1) {
#pragma unroll
          for (int k = 0; k < CPL; ++k)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[k][j] += __shfl_xor_sync(kFull, acc[k][j], o);
          W += __shfl_xor_sync(kFull, W, o);
          const long long lo = __shfl_xor_sync(kFull, last, o);
          last = lo > last ? lo : last;
        }
        if (q == 0) {
#pragma unroll
          for (int k = 0; k < CPL; ++k)
#pragma unroll
            for (int j = 0; j < 4; ++j) sh[wid][4 * (cl + LPP * k) + j] = acc[k][j];
        }
        const float cmx = warp_fmaxf(cmax);
        const bool wany = __any_sync(kFull, any);
        if (lane == 0) {
          sh[wid][2 * DP] = W;
          shl[wid] = last;
          shm[wid][0] = wany ? 1.f : -INFINITY;  // largest weight
          shm[wid][1] = wany ? 1.f : INFINITY;   // smallest weight
          shm[wid][2] = cmx;
        }
        if (!ring_cons_sync(R, phase, A.err, limit)) return false;
        double *rec = A.rec + h.v * stats_stride(DP);
        for (int t = tid; t < DP; t += kRingCons) {
          double tot = 0.0;
          for (int qq = 0; qq < NW; ++qq) tot += sh[qq][t];
          rec[3 + t] = tot;       // sum w' p
          rec[3 + DP + t] = tot;  // sum p over the valid points: the same sum
        }
        if (tid == 0) {
          double w = 0.0;
          long long lst = -1;
          float m0 = -INFINITY, m1 = INFINITY, m2 = 0.f;
          for (int qq = 0; qq < NW; ++qq) {
            w += sh[qq][2 * DP];
            lst = shl[qq] > lst ? shl[qq] : lst;
            m0 = fmaxf(m0, shm[qq][0]);
            m1 = fminf(m1, shm[qq][1]);
            m2 = fmaxf(m2, shm[qq][2]);
          }
          rec[0] = w;  // W
          rec[1] = w;  // valid count
          rec[2] = (double)lst;
          rec[3 + 2 * DP] = m0;
          rec[4 + 2 * DP] = m1;
          rec[5 + 2 * DP] = m2;
        }
        // sh is rewritten by the next chunk's close
        return ring_cons_sync(R, phase, A.err, limit);
      },
      A.err, limit);
}

constexpr size_t ring_sum_smem() { return (size_t)kRingSumStages * kRingSumStageBytes; }

// ---------------------------------------------------------------------------
// Packing of the tensor-core layout (equal weights, no mask): each 64-point
// tile of a side as fp16 hi and lo halves in the core-matrix layout, byte
// (d/8)*1024 + j*16 + (d%8)*2 for point j, coordinate d, and its slot values
// (|x'|^2, |x'|^2 - log2 a, a * weight scale), as packtc_kernel writes them.
// A stage holds the rows of one tile (R = 64) of a chunk's real points -- tile padding past the side's count is not copied
// and packs as zeros -- plus, in a chunk's first stage, the side's anchor
// pairs.  Lane l of a warp packs coordinate group l % NG (8 coordinates) of
// point l / NG of the warp's step: its two float4 reads from shared memory
// are at most 2-way conflicted, and each store instruction writes whole
// 32-byte sectors of the tile (NG groups x 32 / NG consecutive points).
// |x'|^2 is summed over a point's lanes by shuffles.
// ---------------------------------------------------------------------------
template <int DP>
struct RingPackGeom {
  static constexpr int NG = DP / 8;     // coordinate groups per point
  static constexpr int PPI = 32 / NG;   // points per warp step
  static constexpr int R = 64;          // rows per stage: one tile
  static constexpr int NS = DP >= 128 ? 3 : 5;  // stages (~100 KB or less per CTA)
  static constexpr uint32_t OANC = R * DP * 4;
  static constexpr uint32_t SB = (OANC + 2 * DP * 4 + 127) / 128 * 128;
};

template <int DP>
constexpr size_t ring_pack_smem() {
  return (size_t)RingPackGeom<DP>::NS * RingPackGeom<DP>::SB;
}

template <int DP>
__global__ void __launch_bounds__(kRingThreads, 2) packtc_ring_kernel(PrepArgs A,
                                                                      RingRun run) {
  const unsigned limit = run.limit;
  using G = RingPackGeom<DP>;
  constexpr int NS = G::NS, NG = G::NG, PPI = G::PPI, R = G::R;
  constexpr int TB = DP * 128;  // bytes of a hi (or lo) tile
  extern __shared__ __align__(128) uint8_t ring_buf[];
  __shared__ RingCtl<NS> RC;
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int D = A.D;
  ring_init(RC);

  if (wid == kRingProdWarp) {
    if (lane == 0 && !run.idle) {
      const uint32_t k = ring_produce(
          M, RC, smem_u32(ring_buf), G::SB, R,
          [&](RingHdr &h, int64_t &b, int64_t &e) {
            const Seg sg = A.seg[h.p];
            const double *meta = A.meta + h.p * meta_stride(DP);
            h.s = h.side == 0 ? sg.xs : sg.ys;
            h.count = h.side == 0 ? sg.xcount : sg.ycount;
            h.tb = (h.side == 0 ? A.tbase_x : A.tbase_y)[h.p];
            h.k_x = 1.0 / meta[h.side];  // a = 1 / W for every real point
            h.cs = meta[meta_tc_cscale(DP) + h.side];
            h.cc = meta[meta_tc_wscale(DP) + h.side];
            h.scl = pair_scale(A.scale, A.sigma_p, h.p);
            const int64_t cend = ceil_div(h.count, (int64_t)kTile) * kTile;  // through the last tile
            b = h.c * kChunk;
            e = b + kChunk < cend ? b + kChunk : cend;
          },
          [&](RingHdr &h, uint32_t dst, uint32_t bar) {
            const float *pts = h.side == 0 ? A.x : A.y;
            int64_t real = h.count - h.r0;  // rows of the stage that are points
            real = real < 0 ? 0 : (real > h.nr ? h.nr : real);
            const bool anc = (h.flags & kRingFirst) != 0;
            const uint32_t rb = (uint32_t)real * (uint32_t)(D * 4);
            const uint32_t bytes = rb + (anc ? 2u * DP * 4 : 0u);
            if (bytes) mbar_tx(bar, bytes);
            if (rb) bulk_g2s(dst, pts + (h.s + h.r0) * D, rb, bar);
            if (anc) {
              const double *meta = A.meta + h.p * meta_stride(DP);
              bulk_g2s(dst + G::OANC, tc_anchor(meta, DP, h.side), 2u * DP * 4, bar);
            }
          },
          A.err, limit);
      ring_drain(RC, k, kTcSpinLimit);
    }
    return;
  }

  // ---- consumers ----
  const int g = lane % NG;  // this lane's coordinate group (fixed)
  float ah[8], al[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) ah[u] = al[u] = 0.f;
  ring_consume(
      RC, ring_buf, G::SB,
      [&](const RingHdr &h, const uint8_t *st) -> bool {
        if (h.flags & kRingFirst) {
          const float *an = reinterpret_cast<const float *>(st + G::OANC);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            ah[u] = an[8 * g + u];
            al[u] = an[DP + 8 * g + u];
          }
        }
        uint8_t *hp = h.side == 0 ? A.hx : A.hy;
        uint8_t *lp = h.side == 0 ? A.lx : A.ly;
        float *cp = h.side == 0 ? A.cx : A.cy;
        float *Ap = h.side == 0 ? A.Ax : A.Ay;
        const float sc = h.scl, cs = (float)h.cs, wsc = (float)h.cc;
        const float ar = (float)h.k_x;
        const float lga = log2f(ar);  // a is the same for every point of the side
        // a warp-uniform loop (every lane takes part in the shuffles) over two
        // independent sets of points per iteration, loads first
        constexpr int STEP = kRingWarps * PPI;
        for (int base = wid * PPI; base < h.nr; base += 2 * STEP) {
          float xv[2][8];
          bool act[2], real[2];
          int64_t i[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int pi = base + u * STEP + lane / NG;  // point of the stage
            act[u] = pi < h.nr;
            i[u] = h.r0 + pi;  // row of the side
            real[u] = act[u] && i[u] < h.count;
            const float *row = reinterpret_cast<const float *>(st) + (size_t)pi * D;
            if (real[u] && 8 * g + 8 <= D) {
              const float4 r0 = *reinterpret_cast<const float4 *>(row + 8 * g);
              const float4 r1 = *reinterpret_cast<const float4 *>(row + 8 * g + 4);
              const float rv[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
              for (int q = 0; q < 8; ++q) xv[u][q] = sc * ((rv[q] - ah[q]) - al[q]);
            } else {
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const int d = 8 * g + q;
                xv[u][q] = (real[u] && d < D) ? sc * ((row[d] - ah[q]) - al[q]) : 0.f;
              }
            }
          }
          uint32_t hh[2][4], ll[2][4];
          float sq[2] = {0.f, 0.f};
#pragma unroll
          for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              float hv[2], lv[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                hv[e] = tc_hi16(xv[u][2 * c + e] * cs);
                lv[e] = xv[u][2 * c + e] * cs - hv[e];
              }
              // hi has 11 significant bits inside fp16's normal range (the
              // coordinate scale bounds it by 2^15): the conversion is exact
              hh[u][c] = pack_half2(hv[0], hv[1]);
              ll[u][c] = pack_half2(lv[0], lv[1]);
              sq[u] = fmaf(xv[u][2 * c], xv[u][2 * c], sq[u]);
              sq[u] = fmaf(xv[u][2 * c + 1], xv[u][2 * c + 1], sq[u]);
            }
#pragma unroll
          for (int o = NG / 2; o > 0; o >>= 1) {
            sq[0] += __shfl_xor_sync(kFull, sq[0], o);
            sq[1] += __shfl_xor_sync(kFull, sq[1], o);
          }
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            if (!act[u]) continue;
            const int64_t tile = h.tb + i[u] / kTile;
            const int j = (int)(i[u] % kTile);
            const size_t off = (size_t)tile * TB + (size_t)g * 1024 + (size_t)j * 16;
            *reinterpret_cast<uint4 *>(hp + off) =
                make_uint4(hh[u][0], hh[u][1], hh[u][2], hh[u][3]);
            *reinterpret_cast<uint4 *>(lp + off) =
                make_uint4(ll[u][0], ll[u][1], ll[u][2], ll[u][3]);
            if (g == 0) {
              const float a = real[u] ? ar : 0.f;
              if (real[u]) Ap[h.s + i[u]] = a;
              float *cv = cp + tile * (3 * kTile);
              cv[j] = sq[u];
              cv[kTile + j] = a > 0.f ? sq[u] - lga : INFINITY;
              cv[2 * kTile + j] = a * wsc;
            }
          }
        }
        return true;
      },
      A.err, limit);
}

// ---------------------------------------------------------------------------
// Backward, write pass of the tensor-core layout (the points themselves in,
// packed here; float4 rows; no mask, no weight gradients): per point
//   dL/dx_d = -a k_x (c_s (x'_d s_self - T_self,d) + c_c (x'_d s_cross - T_cross,d))
//             [- a R_d when centred]
// as epigw_write_kernel computes it, term for term.  A stage holds R points:
// their per-point sum records (gen_acc_stride(DP) floats each), their
// coordinates, an aligned run of the workspace's weights around theirs and,
// in a chunk's first stage, the side's fp32 anchor pairs.  A consumer thread
// keeps one float4 coordinate chunk (cc = thread % (DP / 4)) of KR points
// per stage; the gradients go out as coalesced float4 stores.
// ---------------------------------------------------------------------------
constexpr int kRingWriteStages = 4;
constexpr int kRingWriteKR = 2;  // points per consumer thread per stage

template <int DP>
struct RingWriteGeom {
  static constexpr int NC = DP / 4;
  static constexpr int R = kRingWriteKR * kRingCons / NC;  // points per stage
  static constexpr uint32_t ACCB = (uint32_t)gen_acc_stride(DP) * 4;
  static constexpr uint32_t OPTS = R * ACCB;
  static constexpr uint32_t OA = OPTS + R * DP * 4;
  static constexpr uint32_t OANC = OA + R * 4 + 32;  // room for the weights' alignment
  static constexpr uint32_t SB = (OANC + 2 * DP * 4 + 127) / 128 * 128;
  static_assert(ACCB % 16 == 0 && OPTS % 16 == 0 && OA % 16 == 0 && OANC % 16 == 0,
                "stage arrays must start on 16-byte boundaries");
};

template <int DP>
constexpr size_t ring_write_smem() {
  return (size_t)kRingWriteStages * RingWriteGeom<DP>::SB;
}

template <int DP>
__global__ void __launch_bounds__(kRingThreads, 2) epigw_ring_write_kernel(EpilogueArgs A,
                                                                           RingRun run) {
  const unsigned limit = run.limit;
  using G = RingWriteGeom<DP>;
  constexpr int NS = kRingWriteStages, NC = G::NC, R = G::R;
  extern __shared__ __align__(128) uint8_t ring_buf[];
  __shared__ RingCtl<NS> RC;
  const ChunkMap M{A.P, A.choff, A.chx, A.cpair, A.ticket};
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int D = A.D, rs = stats_stride(DP);
  ring_init(RC);

  if (wid == kRingProdWarp) {
    if (lane == 0 && !run.idle) {
      const uint32_t k = ring_produce(
          M, RC, smem_u32(ring_buf), G::SB, R,
          [&](RingHdr &h, int64_t &b, int64_t &e) {
            const EpiSide E = epi_side(A, h.p, h.side);
            h.s = E.s;
            h.count = E.count;
            h.k_x = E.k_x;
            h.cs = E.cs;
            h.cc = E.cc;
            h.scl = side_scale(A, h.p);
            b = h.c * kChunk;
            e = b + kChunk < E.span ? b + kChunk : E.span;
          },
          [&](RingHdr &h, uint32_t dst, uint32_t bar) {
            const float *accb = h.side == 0 ? A.accX : A.accY;
            const float *pts = h.side == 0 ? A.x : A.y;
            const float *Ap = h.side == 0 ? A.Ax : A.Ay;
            const uint32_t nr = (uint32_t)h.nr;
            // the weights from the 16-byte boundary at or below the first one
            // (the workspace pads every array to 256 bytes: in bounds)
            const uintptr_t wa = reinterpret_cast<uintptr_t>(Ap + h.s + h.r0);
            const uintptr_t w0 = wa & ~(uintptr_t)15;
            h.aoff = (int)(wa - w0);
            const uint32_t wbytes = ((uint32_t)h.aoff + nr * 4 + 15u) & ~15u;
            const bool anc = (h.flags & kRingFirst) != 0;
            const uint32_t bytes = nr * G::ACCB + nr * (uint32_t)(D * 4) + wbytes +
                                   (anc ? 2u * DP * 4 : 0u);
            mbar_tx(bar, bytes);
            bulk_g2s(dst, accb + (h.s + h.r0) * A.acc_stride, nr * G::ACCB, bar);
            bulk_g2s(dst + G::OPTS, pts + (h.s + h.r0) * D, nr * (uint32_t)(D * 4), bar);
            bulk_g2s(dst + G::OA, reinterpret_cast<const void *>(w0), wbytes, bar);
            if (anc) bulk_g2s(dst + G::OANC, side_anchor(A, h.p, h.side), 2u * DP * 4, bar);
          },
          A.err, limit);
      ring_drain(RC, k, kTcSpinLimit);
    }
    return;
  }

  // ---- consumers ----
  const int cc = tid % NC;          // this thread's coordinate chunk (fixed)
  const bool has = 4 * cc < D;      // it holds coordinates
  float ah[4] = {0.f, 0.f, 0.f, 0.f}, al[4] = {0.f, 0.f, 0.f, 0.f};
  double Rv[4] = {0.0, 0.0, 0.0, 0.0};
  ring_consume(
      RC, ring_buf, G::SB,
      [&](const RingHdr &h, const uint8_t *st) -> bool {
        if (h.flags & kRingFirst) {
          const float *an = reinterpret_cast<const float *>(st + G::OANC);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            ah[v] = has ? an[4 * cc + v] : 0.f;
            al[v] = has ? an[DP + 4 * cc + v] : 0.f;
            Rv[v] = 0.0;
          }
          if (A.center && has) {
            // the side's totals R_d, summed over its chunks in order
            for (int64_t kk = 0; kk < h.n; ++kk) {
              const double *rc = A.rec + (h.first + kk) * rs + 1 + 4 * cc;
#pragma unroll
              for (int v = 0; v < 4; ++v) Rv[v] += rc[v];
            }
          }
        }
        float *gout = h.side == 0 ? A.grad_x : A.grad_y;
        if (gout == nullptr || !has) return true;
        const float *aw = reinterpret_cast<const float *>(st + G::OA + h.aoff);
#pragma unroll
        for (int j = 0; j < kRingWriteKR; ++j) {
          const int i = (tid + j * kRingCons) / NC;  // point of the stage
          if (i >= h.nr) break;
          const int64_t row = h.r0 + i;
          const int64_t g = h.s + row;
          float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
          if (row < h.count) {
            const float *accr = reinterpret_cast<const float *>(st + (size_t)i * G::ACCB);
            const float4 ts = *reinterpret_cast<const float4 *>(accr + 4 * cc);
            const float4 tc = *reinterpret_cast<const float4 *>(accr + DP + 4 * cc);
            const double s_self = accr[2 * DP], s_cross = accr[2 * DP + 1];
            const float4 r = *reinterpret_cast<const float4 *>(
                st + G::OPTS + (size_t)i * (D * 4) + 16 * cc);
            const double a = aw[i];
            const float xv[4] = {h.scl * ((r.x - ah[0]) - al[0]), h.scl * ((r.y - ah[1]) - al[1]),
                                 h.scl * ((r.z - ah[2]) - al[2]), h.scl * ((r.w - ah[3]) - al[3])};
            const float tsv[4] = {ts.x, ts.y, ts.z, ts.w};
            const float tcv[4] = {tc.x, tc.y, tc.z, tc.w};
            float rr[4];
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const double Gs = xv[v] * s_self - (double)tsv[v];
              const double Gc = xv[v] * s_cross - (double)tcv[v];
              double gx = -a * h.k_x * (h.cs * Gs + h.cc * Gc);
              if (A.center) gx -= a * Rv[v];
              rr[v] = (float)gx;
            }
            o = make_float4(rr[0], rr[1], rr[2], rr[3]);
          }
          *reinterpret_cast<float4 *>(gout + g * D + 4 * cc) = o;
        }
        return true;
      },
      A.err, limit);
}

}  // namespace ra
