// ra_chunks.cuh -- work decomposition of the O(N) passes (weight and centroid
// sums, packing, the backward epilogue).
//
// Each side of each pair is cut into chunks of kChunk points.  Pair p owns
// the virtual chunks [choff[p], choff[p + 1]): the first chx[p] of them cover
// its x points, the rest its y points.  A pass launches a fixed grid; CTA b
// walks the contiguous virtual range [b * per, (b + 1) * per), so a huge pair
// spreads over many SMs while a batch of small pairs costs one CTA visit per
// chunk.  Partial sums are stored per virtual chunk and combined per pair in
// chunk order, which keeps every result independent of scheduling.
//
// With a chunk ticket (ChunkMap::ticket, zeroed before the launch) the CTAs
// instead take chunks one at a time from a shared counter, each chunk's pair
// read from cpair[v]: chunks differ in size by up to kChunk / 32 (a batch of
// graphs of 32-1024 points), and a fixed range of them per CTA leaves the
// slowest CTA with about half again the mean work.
#pragma once

#include "ra_common.cuh"

namespace ra {

constexpr int kChunk = 1024;  // points per chunk (a multiple of kTile)
static_assert(kChunk % kTile == 0, "a chunk must hold whole tiles");

// One step of a block-wide inclusive scan (sum or max) over 1024 values, one
// per thread of a CTA of 1024; `carry` (shared) holds the result of the
// previous steps and is advanced.  Called by all threads.
template <bool MAX>
__device__ __forceinline__ int64_t block_scan_step(int64_t v, int64_t *warp_tot,
                                                   int64_t *carry) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  int64_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t t = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl = MAX ? (t > incl ? t : incl) : incl + t;
  }
  if (lane == 31) warp_tot[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    int64_t t = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t u = __shfl_up_sync(kFull, t, o);
      if (lane >= o) t = MAX ? (u > t ? u : t) : t + u;
    }
    warp_tot[lane] = t;  // inclusive over warps
  }
  __syncthreads();
  int64_t r = incl;
  if (wid > 0) r = MAX ? (warp_tot[wid - 1] > r ? warp_tot[wid - 1] : r) : r + warp_tot[wid - 1];
  r = MAX ? (*carry > r ? *carry : r) : r + *carry;
  __syncthreads();
  if (tid == 1023) *carry = r;
  __syncthreads();
  return r;
}

// Block-wide exclusive scan of src[0, n) into dst[0, n] (dst[n] = total),
// every prefix clamped to `cap`.  Called by all threads of one CTA of 1024.
__device__ __forceinline__ void block_exclusive_scan(const int64_t *src, int64_t *dst, int64_t n,
                                                     int64_t cap, int64_t *warp_tot,
                                                     int64_t *carry) {
  if (threadIdx.x == 0) *carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < n; base += 1024) {
    const int64_t i = base + threadIdx.x;
    const int64_t v = i < n ? src[i] : 0;
    const int64_t incl = block_scan_step<false>(v, warp_tot, carry);
    if (i < n) {
      const int64_t e = incl - v;
      dst[i] = e < cap ? e : cap;
    }
  }
  if (threadIdx.x == 0) dst[n] = *carry < cap ? *carry : cap;
  __syncthreads();
}

struct ChunkMap {
  int64_t P;
  const int64_t *choff;  // [P + 1], clamped to the workspace bound
  const int64_t *chx;    // [P]: chunks of the x side
  const int32_t *cpair = nullptr;  // [choff[P]]: the pair of each virtual chunk
  unsigned *ticket = nullptr;      // chunk counter of this launch (null: fixed ranges)
};

// Largest p in [0, P) with choff[p] <= v (v < choff[P]).
__device__ __forceinline__ int64_t chunk_pair(const ChunkMap &M, int64_t v) {
  int64_t lo = 0, hi = M.P;
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (M.choff[mid] <= v) lo = mid;
    else hi = mid;
  }
  return lo;
}

// Runs f(p, side, c, v, first, n) for every virtual chunk v of this CTA's
// range: chunk c of the side's n chunks, whose records start at virtual index
// `first`.  The range and all arguments are uniform over the CTA, so f may
// synchronise the block.
// Pair tickets for the one-CTA-per-pair kernels, in a for loop's three parts:
//   for (p = pair_ticket_first(ctr, slot); p < P; p = pair_ticket_next(slot, ++k, nxt)) {
//     nxt = pair_ticket_take(ctr);  // the next pair, fetched while this one runs
//     ...                           // `continue` still reaches the barrier
//   }
// Thread 0 draws; the CTA reads the draw after a barrier, from two slots (a
// slot is rewritten only two barriers after it was read).  Pairs differ in
// size by up to 64x (a batch of graphs of 32-2048 points), and a fixed
// round-robin share per CTA left the slowest CTA with ~40 % more work than
// the mean.
__device__ __forceinline__ int64_t pair_ticket_first(unsigned *ctr, unsigned *slot) {
  if (threadIdx.x == 0) slot[0] = atomicAdd(ctr, 1u);
  __syncthreads();
  return slot[0];
}
__device__ __forceinline__ unsigned pair_ticket_take(unsigned *ctr) {
  return threadIdx.x == 0 ? atomicAdd(ctr, 1u) : 0u;
}
__device__ __forceinline__ int64_t pair_ticket_next(unsigned *slot, int k, unsigned nxt) {
  if (threadIdx.x == 0) slot[k & 1] = nxt;
  __syncthreads();
  return slot[k & 1];
}

template <typename F>
__device__ __forceinline__ void for_each_chunk(const ChunkMap &M, F &&f) {
  const int64_t total = M.choff[M.P];
  if (M.ticket != nullptr && M.cpair != nullptr) {
    // one chunk per ticket; thread 0 takes the next ticket while the current
    // chunk runs, and publishes it in the other of two slots before the
    // barrier that ends the chunk (a slot is rewritten only two barriers
    // after it was read)
    __shared__ unsigned fec_slot[2];
    if (threadIdx.x == 0) fec_slot[0] = atomicAdd(M.ticket, 1u);
    __syncthreads();
    unsigned cur = fec_slot[0];
    for (int k = 1; (int64_t)cur < total; ++k) {
      unsigned nxt = 0;
      if (threadIdx.x == 0) nxt = atomicAdd(M.ticket, 1u);
      const int64_t v = cur;
      const int64_t p = M.cpair[v];
      const int64_t lo = M.choff[p], hi = M.choff[p + 1];
      int64_t cx = M.chx[p];
      if (cx > hi - lo) cx = hi - lo;
      const int64_t local = v - lo;
      const int side = local < cx ? 0 : 1;
      const int64_t c = side == 0 ? local : local - cx;
      const int64_t first = side == 0 ? lo : lo + cx;
      const int64_t n = side == 0 ? cx : (hi - lo) - cx;
      f(p, side, c, v, first, n);
      if (threadIdx.x == 0) fec_slot[k & 1] = nxt;
      __syncthreads();
      cur = fec_slot[k & 1];
    }
    return;
  }
  const int64_t per = ceil_div(total, (int64_t)gridDim.x);
  int64_t v = (int64_t)blockIdx.x * per;
  const int64_t v1 = v + per < total ? v + per : total;
  if (v >= v1) return;
  int64_t p = chunk_pair(M, v);
  int64_t lo = M.choff[p], hi = M.choff[p + 1];
  for (; v < v1; ++v) {
    while (v >= hi) {
      ++p;
      lo = hi;
      hi = M.choff[p + 1];
    }
    int64_t cx = M.chx[p];
    if (cx > hi - lo) cx = hi - lo;  // only a malformed ptr truncates the map
    const int64_t local = v - lo;
    const int side = local < cx ? 0 : 1;
    const int64_t c = side == 0 ? local : local - cx;
    const int64_t first = side == 0 ? lo : lo + cx;
    const int64_t n = side == 0 ? cx : (hi - lo) - cx;
    f(p, side, c, v, first, n);
  }
}

}  // namespace ra
