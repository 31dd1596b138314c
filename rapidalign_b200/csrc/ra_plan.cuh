// ra_plan.cuh -- device-side work planning: per-pair item counts, an exclusive
// scan over pairs and the emission of the item list.  Everything stays on the
// device, so a forward needs no host round trip to size its work.
#pragma once

#include "ra_common.cuh"

namespace ra {

struct PlanArgs {
  int64_t P;
  int generic;        // 0: D <= 3 tiles (3 blocks), 1: generic rows (4 orientations),
                      // 2: D <= 3 tiles, both orientations, rows only (deterministic mode)
  const Seg *seg;
  int64_t *cnt;       // [P]: items of pair p
  int64_t *boff;      // [P * 4]: local start of each block inside the pair's items
  int64_t *item_off;  // [P + 1]
  int64_t *n_items;   // device scalar (== item_off[P])
  Item *items;
  int64_t max_items;  // capacity of `items` (the host bound)
  // D <= 3 tiles: the order the tile kernel takes the items in (null: plan
  // order): pairs by decreasing size, each pair's items contiguous and in
  // plan order.  hist (items per size bucket), cursor and bbase (first
  // position of a bucket): [kSizeBuckets] counters, zeroed before the plan.
  int32_t *order;
  int32_t *hist, *cursor, *bbase;
};

constexpr int kSizeBuckets = 256;

// A pair's size bucket: 64-point tiles of its larger side, capped.
__device__ __forceinline__ int pair_size_key(const Seg &s) {
  const int64_t n = s.xcount > s.ycount ? s.xcount : s.ycount;
  const int64_t t = ceil_div(n, (int64_t)kTile);
  return t > kSizeBuckets - 1 ? kSizeBuckets - 1 : (int)t;
}

__device__ __forceinline__ void block_counts(const Seg &s, int generic, int64_t c[4]) {
  if (generic == 2) {
    const int64_t nTx = ceil_div(s.xcount, (int64_t)kTile);
    const int64_t nTy = ceil_div(s.ycount, (int64_t)kTile);
    c[0] = nTx;  // x rows vs y cols
    c[1] = nTx;  // x vs x
    c[2] = nTy;  // y vs y
    c[3] = nTy;  // y rows vs x cols
  } else if (!generic) {
    const int64_t nTx = ceil_div(s.xcount, (int64_t)kTile);
    const int64_t nTy = ceil_div(s.ycount, (int64_t)kTile);
    c[0] = nTx * splits_for(nTy);  // x rows vs y cols
    c[1] = nTx * splits_for(nTx);  // x vs x
    c[2] = nTy * splits_for(nTy);  // y vs y
    c[3] = 0;
  } else {
    const int64_t nRx = ceil_div(s.xcount, (int64_t)kGenRows);
    const int64_t nRy = ceil_div(s.ycount, (int64_t)kGenRows);
    c[0] = nRx;  // x vs y
    c[1] = nRx;  // x vs x
    c[2] = nRy;  // y vs y
    c[3] = nRy;  // y vs x
  }
}

__global__ void plan_count_kernel(PlanArgs A) {
  const int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (p >= A.P) return;
  int64_t c[4];
  const Seg sg = A.seg[p];
  block_counts(sg, A.generic, c);
  A.boff[p * 4 + 0] = 0;
  A.boff[p * 4 + 1] = c[0];
  A.boff[p * 4 + 2] = c[0] + c[1];
  A.boff[p * 4 + 3] = c[0] + c[1] + c[2];
  A.cnt[p] = c[0] + c[1] + c[2] + c[3];
  if (A.order != nullptr && A.cnt[p] > 0) atomicAdd(&A.hist[pair_size_key(sg)], (int)A.cnt[p]);
}

// Exclusive scan of the per-pair item counts into item_off ([P + 1]); one
// CTA of 1024 threads.  (The D <= 3 tile bases are scanned by segment_kernel.)
__global__ void __launch_bounds__(1024) plan_scan_kernel(PlanArgs A) {
  __shared__ int64_t warp_tot[32];
  __shared__ int64_t carry_sh;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  {
    const int64_t *src = A.cnt;
    int64_t *dst = A.item_off;
    if (tid == 0) carry_sh = 0;
    __syncthreads();
    for (int64_t base = 0; base < A.P; base += 1024) {
      const int64_t i = base + tid;
      const int64_t v = i < A.P ? src[i] : 0;
      int64_t incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t n = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += n;
      }
      if (lane == 31) warp_tot[wid] = incl;
      __syncthreads();
      if (wid == 0) {
        int64_t t = warp_tot[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int64_t n = __shfl_up_sync(kFull, t, o);
          if (lane >= o) t += n;
        }
        warp_tot[lane] = t;  // inclusive over warps
      }
      __syncthreads();
      const int64_t before = carry_sh + (wid > 0 ? warp_tot[wid - 1] : 0);
      if (i < A.P) dst[i] = before + incl - v;
      __syncthreads();
      if (tid == 1023) carry_sh = before + incl;
      __syncthreads();
    }
    if (tid == 0) {
      int64_t tot = carry_sh;
      if (tot > A.max_items) tot = A.max_items;  // cannot happen with the host bound
      *A.n_items = tot;
      dst[A.P] = tot;
    }
  }
  if (A.order != nullptr) {
    // first position of each size bucket, the largest pairs first
    __shared__ int32_t hs[kSizeBuckets];
    for (int b = tid; b < kSizeBuckets; b += blockDim.x) hs[b] = A.hist[b];
    __syncthreads();
    if (tid == 0) {
      int32_t run = 0;
      for (int b = kSizeBuckets - 1; b >= 0; --b) {
        A.bbase[b] = run;
        run += hs[b];
      }
    }
  }
}

// One CTA per pair writes that pair's items.
__global__ void plan_emit_kernel(PlanArgs A) {
  const int64_t p = blockIdx.x;
  if (p >= A.P) return;
  const Seg s = A.seg[p];
  int64_t c[4];
  block_counts(s, A.generic, c);
  const int64_t base = A.item_off[p];
  const int64_t total = c[0] + c[1] + c[2] + c[3];
  int64_t S[4] = {1, 1, 1, 1};
  if (A.generic == 0) {
    const int64_t nTx = ceil_div(s.xcount, (int64_t)kTile);
    const int64_t nTy = ceil_div(s.ycount, (int64_t)kTile);
    S[0] = splits_for(nTy);
    S[1] = splits_for(nTx);
    S[2] = splits_for(nTy);
  }
  for (int64_t l = threadIdx.x; l < total; l += blockDim.x) {
    if (base + l >= A.max_items) break;
    int b = 0;
    int64_t loc = l;
    while (b < 3 && loc >= c[b]) {
      loc -= c[b];
      ++b;
    }
    Item it;
    it.pair = (int)p;
    it.block = b;
    // split-major, row tiles fastest: a split evaluation that deals items out
    // round-robin (item % shard_count) then gives every shard an equal share
    // of each split's row tiles -- in self blocks the late splits hold most of
    // the work -- and consecutive tickets read the same column tiles
    const int64_t nr = c[b] / S[b];  // row tiles of this block
    it.tile = (int)(loc % nr);
    it.split = (int)(loc / nr);
    A.items[base + l] = it;
  }
  if (A.order != nullptr && total > 0) {
    // the pair's items take one contiguous run of the order, in plan order,
    // at a place in their size bucket (pairs of one bucket in any order:
    // every item writes its own partials, reduced later in plan order)
    __shared__ int64_t pos;
    if (threadIdx.x == 0)
      pos = (int64_t)A.bbase[pair_size_key(s)] + atomicAdd(&A.cursor[pair_size_key(s)], (int)total);
    __syncthreads();
    for (int64_t l = threadIdx.x; l < total; l += blockDim.x)
      if (pos + l < A.max_items && base + l < A.max_items) A.order[pos + l] = (int32_t)(base + l);
  }
}

}  // namespace ra
