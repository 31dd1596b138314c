// ra_capi.cu -- host side of the C ABI declared in include/rapidalign_b200.h.
// Lays out the caller's workspace, validates arguments and enqueues the
// kernel pipeline on the caller's stream:
//   segments + chunk map -> stats (per chunk) -> meta (per pair) ->
//   [generic pack] -> plan count -> plan scan -> plan emit -> [tile pack] ->
//   tiles -> finalize (per pair)                                 [forward]
//   epilogue partials (per chunk) -> epilogue write (per chunk)  [backward]
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>

#include "../../include/rapidalign_b200.h"
#include "ra_batch.cuh"
#include "ra_chunks.cuh"
#include "ra_common.cuh"
#include "ra_epilogue.cuh"
#include "ra_exact.cuh"
#include "ra_pdl.cuh"
#include "ra_plan.cuh"
#include "ra_prep.cuh"
#include "ra_ring.cuh"
#include "ra_tc16.cuh"
#include "ra_tiles3.cuh"
#include "ra_tilesg.cuh"

namespace {

using namespace ra;

std::atomic<unsigned long long> g_launches{0};

constexpr int kPrepThreads = 256;
constexpr int kEpiThreads = 256;
constexpr int kChunkCtasPerSm = 8;  // 256-thread CTAs of the per-chunk passes

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

int generic_dp(int D) {
  int r = 4;
  while (r < D) r <<= 1;
  return r;
}

struct Layout {
  bool packed3;
  bool tc16;        // generic layout on the tensor cores: fp16 tiles (ra_tc16.cuh)
  int DP;
  int nq;           // packed3: 16-byte arrays per tile
  int acc_stride;
  int64_t max_items;
  int64_t max_tiles_x, max_tiles_y;  // packed3: bound on the padded tiles
  int64_t max_chunks;                // bound on the virtual chunks (ra_chunks.cuh)
  size_t hdr, seg, meta, cnt, item_off, tbase_x, tbase_y, boff, items, itemK, itemS, Kws, Sws,
      coef, Ktmp, chcnt, chx, choff, rec, cpair;
  size_t tiles_x, tiles_y, Gx, Gy, Ax, Ay, accX, accY;
  size_t hx, hy, lx, ly, cx, cy;  // tc16: fp16 hi / lo tiles and slot values
  size_t ix;                      // tc16: one ItemX record per work item
  size_t order;                   // packed3: the tile kernel's item order (ra_plan.cuh)
  size_t acc_x_bytes, acc_y_bytes;
  size_t total;
};

// header block: int err @0, unsigned ticket @4, int has_state @8, int64 n_items @16,
// unsigned chunk tickets @32 (ra_chunks.cuh): [0] the sums pass, [1] packing,
// [2] [3] the backward's partial and write passes; pair tickets: [4]
// prep3_kernel, [5] epi3_small_kernel
constexpr size_t kHdrErr = 0, kHdrTicket = 4, kHdrState = 8, kHdrNItems = 16,
                 kHdrChunkTickets = 32;
// then the item order's size-bucket counters (ra_plan.cuh): hist @256,
// cursor @256 + 4 kSizeBuckets, bbase @256 + 8 kSizeBuckets; the whole
// header is zeroed at the start of every forward
constexpr size_t kHdrSizeHist = 256, kHdrBytes = 4096;
static_assert(kHdrSizeHist + 3 * 4 * kSizeBuckets <= kHdrBytes, "header too small");
constexpr int kItemF64 = 2;  // fp64 partials per work item: K, S

bool desc_ok(const ra_kde_desc *d) {
  if (d == nullptr) return false;
  if (d->num_pairs < 0 || d->dim < 1 || d->dim > 256) return false;
  if (d->layout != RA_LAYOUT_RAGGED && d->layout != RA_LAYOUT_DENSE) return false;
  if (d->num_x < 0 || d->num_y < 0) return false;
  if (d->layout == RA_LAYOUT_DENSE) {
    if (d->nmax_x < 0 || d->nmax_y < 0) return false;
    if (d->num_x != d->num_pairs * d->nmax_x || d->num_y != d->num_pairs * d->nmax_y)
      return false;
  }
  if (d->weights_x < 0 || d->weights_x > 3 || d->weights_y < 0 || d->weights_y > 3) return false;
  if (d->num_x > ((int64_t)1 << 40) || d->num_y > ((int64_t)1 << 40)) return false;
  if (d->num_pairs > ((int64_t)1 << 30)) return false;
  if (d->engine < RA_ENGINE_AUTO || d->engine > RA_ENGINE_TENSOR) return false;
  if (d->engine == RA_ENGINE_TENSOR && d->dim > 3) {
    const int dp = generic_dp(d->dim);
    if (dp != 32 && dp != 64 && dp != 128) return false;
  }
  if (d->shard_count < 0 || (d->shard_count > 1 &&
                             (d->shard_index < 0 || d->shard_index >= d->shard_count)))
    return false;
  if ((d->test_hooks & ~(RA_TEST_NO_MMA | RA_TEST_RING_IDLE)) != 0) return false;
  if (d->skip_weight_sums != 0 && d->skip_weight_sums != 1) return false;
  if (d->deterministic != 0 && d->deterministic != 1) return false;
  return true;
}

bool use_tensor_cores(const ra_kde_desc *d, int DP) {
  if (d->dim <= 3 || d->engine == RA_ENGINE_SIMT) return false;
  return DP == 32 || DP == 64 || DP == 128;
}

Layout make_layout(const ra_kde_desc *d) {
  Layout L;
  std::memset(&L, 0, sizeof(L));
  const int64_t P = d->num_pairs, NX = d->num_x, NY = d->num_y;
  L.packed3 = d->dim <= 3;
  L.DP = L.packed3 ? 3 : generic_dp(d->dim);
  L.tc16 = !L.packed3 && use_tensor_cores(d, L.DP);
  L.acc_stride = L.packed3 ? kAcc3Stride : gen_acc_stride(L.DP);
  // host bound on the number of items
  int64_t tx, ty;  // sum over pairs of row tiles
  const int64_t rows = L.packed3 ? kTile : kGenRows;
  if (d->layout == RA_LAYOUT_DENSE) {
    tx = P * ceil_div(d->nmax_x, rows);
    ty = P * ceil_div(d->nmax_y, rows);
  } else {
    tx = ceil_div(NX, rows) + P;
    ty = ceil_div(NY, rows) + P;
  }
  L.max_items = L.packed3 ? (int64_t)kSplitMax * (2 * tx + ty) : 2 * tx + 2 * ty;
  if (L.max_items < 1) L.max_items = 1;
  if (d->layout == RA_LAYOUT_DENSE)
    L.max_chunks = P * (ceil_div(d->nmax_x, kChunk) + ceil_div(d->nmax_y, kChunk));
  else
    L.max_chunks = ceil_div(NX, kChunk) + ceil_div(NY, kChunk) + 2 * P;
  if (L.max_chunks < 1) L.max_chunks = 1;
  L.max_tiles_x = L.packed3 ? (tx > 0 ? tx : 1) : 0;
  L.max_tiles_y = L.packed3 ? (ty > 0 ? ty : 1) : 0;
  if (L.tc16) {
    // 64-point tiles of the fp16 layout: room for every pair's span
    const int64_t t64x = d->layout == RA_LAYOUT_DENSE ? P * ceil_div(d->nmax_x, (int64_t)kTile)
                                                      : ceil_div(NX, (int64_t)kTile) + P;
    const int64_t t64y = d->layout == RA_LAYOUT_DENSE ? P * ceil_div(d->nmax_y, (int64_t)kTile)
                                                      : ceil_div(NY, (int64_t)kTile) + P;
    L.max_tiles_x = t64x > 0 ? t64x : 1;
    L.max_tiles_y = t64y > 0 ? t64y : 1;
  }
  const bool grad = d->need_grad != 0;
  L.nq = kT3Arrays;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o = a256(o + bytes);
    return at;
  };
  const size_t P1 = (size_t)(P > 0 ? P : 1);
  L.hdr = take(kHdrBytes);
  L.seg = take(sizeof(Seg) * P1);
  L.meta = take(sizeof(double) * P1 * meta_stride(L.DP));
  L.cnt = take(sizeof(int64_t) * 3 * P1);
  L.item_off = take(sizeof(int64_t) * (P1 + 1));
  L.tbase_x = take(sizeof(int64_t) * (P1 + 1));
  L.tbase_y = take(sizeof(int64_t) * (P1 + 1));
  L.boff = take(sizeof(int64_t) * 4 * P1);
  L.items = take(sizeof(Item) * (size_t)L.max_items);
  // itemK and itemS form one contiguous fp64 region of kItemF64 values per
  // item (reduced across shards)
  L.itemK = take(sizeof(double) * kItemF64 * (size_t)L.max_items);
  L.itemS = L.itemK + sizeof(double) * (size_t)L.max_items;
  L.Kws = take(sizeof(double) * 3 * P1);
  L.Sws = take(sizeof(double) * 3 * P1);
  L.coef = take(sizeof(double) * 3 * P1);
  L.Ktmp = take(sizeof(double) * 3 * P1);
  L.chcnt = take(sizeof(int64_t) * P1);
  L.chx = take(sizeof(int64_t) * P1);
  L.choff = take(sizeof(int64_t) * (P1 + 1));
  L.rec = take(sizeof(double) * (size_t)L.max_chunks * stats_stride(L.DP));
  L.cpair = take(sizeof(int32_t) * (size_t)L.max_chunks);
  const size_t nx = (size_t)(NX > 0 ? NX : 1), ny = (size_t)(NY > 0 ? NY : 1);
  if (L.packed3) {
    L.order = take(sizeof(int32_t) * (size_t)L.max_items);
    L.tiles_x = take((size_t)16 * L.nq * kTile * (size_t)L.max_tiles_x);
    L.tiles_y = take((size_t)16 * L.nq * kTile * (size_t)L.max_tiles_y);
    L.Ax = take(sizeof(float) * kTile * (size_t)L.max_tiles_x);  // a~ per slot
    L.Ay = take(sizeof(float) * kTile * (size_t)L.max_tiles_y);
    L.acc_x_bytes = sizeof(float) * kAcc3Stride * kTile * (size_t)L.max_tiles_x;
    L.acc_y_bytes = sizeof(float) * kAcc3Stride * kTile * (size_t)L.max_tiles_y;
  } else {
    L.Gx = take(sizeof(float) * nx * L.DP);
    L.Gy = take(sizeof(float) * ny * L.DP);
    L.Ax = take(sizeof(float) * nx);
    L.Ay = take(sizeof(float) * ny);
    if (L.tc16) {
      const size_t tbytes = (size_t)t16_tile_bytes(L.DP);
      L.hx = take(tbytes * (size_t)L.max_tiles_x);
      L.lx = take(tbytes * (size_t)L.max_tiles_x);
      L.hy = take(tbytes * (size_t)L.max_tiles_y);
      L.ly = take(tbytes * (size_t)L.max_tiles_y);
      L.cx = take(sizeof(float) * kT16SlotFloats * (size_t)L.max_tiles_x);
      L.cy = take(sizeof(float) * kT16SlotFloats * (size_t)L.max_tiles_y);
      L.ix = take(sizeof(ItemX) * (size_t)L.max_items);
    }
    L.acc_x_bytes = sizeof(float) * nx * L.acc_stride;
    L.acc_y_bytes = sizeof(float) * ny * L.acc_stride;
  }
  if (grad) {
    L.accX = take(L.acc_x_bytes);
    L.accY = take(L.acc_y_bytes);
  }
  L.total = o;
  return L;
}

template <typename T>
T *at(void *ws, size_t off) {
  return reinterpret_cast<T *>(static_cast<char *>(ws) + off);
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? RA_OK : RA_ERR_CUDA; }

float scale_for(double sigma) { return scale_of_sigma(sigma); }

int check_common(const ra_kde_desc *d, void *ws, size_t ws_bytes, size_t need) {
  if (!desc_ok(d)) return RA_ERR_INVALID_ARGUMENT;
  if (!(d->sigma > 0.0) || !std::isfinite(d->sigma)) return RA_ERR_SIGMA;
  if (ws == nullptr || ((uintptr_t)ws & 255) != 0 || ws_bytes < need) return RA_ERR_WORKSPACE;
  return RA_OK;
}

// Grid of the per-chunk passes: enough CTAs to fill the GPU, never more than
// there can be chunks.
// 16-byte vector loads and stores of caller memory need 16-byte aligned
// pointers (a contiguous tensor can start at any float); null counts as
// aligned.
bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The ring passes' wait bound (RA_TEST_RING_IDLE: idle producers and short
// waits, for the failure-path tests).
RingRun ring_run(const ra_kde_desc *d) {
  RingRun r;
  const bool idle = (d->test_hooks & RA_TEST_RING_IDLE) != 0;
  r.limit = idle ? 4096u : kTcSpinLimit;
  r.idle = idle ? 1 : 0;
  return r;
}

// The sums pass on the bulk-copy ring: two CTAs per SM (dynamic shared
// memory above the 48 KB default).
template <int DP>
int launch_statsw_ring_d(const PrepArgs &pa, const RingRun &run, cudaStream_t st) {
  const size_t smem = ring_sum_smem();
  if (cudaFuncSetAttribute(statsw_ring_kernel<DP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return RA_ERR_CUDA;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  statsw_ring_kernel<DP><<<(unsigned)(sms > 0 ? 2 * sms : 2), kRingThreads, smem, st>>>(
      pa, run);
  return RA_OK;
}
template <int DP>
int launch_write_ring_d(const EpilogueArgs &ea, const RingRun &run, cudaStream_t st) {
  const size_t smem = ring_write_smem<DP>();
  if (cudaFuncSetAttribute(epigw_ring_write_kernel<DP>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return RA_ERR_CUDA;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  epigw_ring_write_kernel<DP><<<(unsigned)(sms > 0 ? 2 * sms : 2), kRingThreads, smem, st>>>(
      ea, run);
  return RA_OK;
}
int launch_write_ring(int DP, const EpilogueArgs &ea, const RingRun &run, cudaStream_t st) {
  if (DP == 32) return launch_write_ring_d<32>(ea, run, st);
  if (DP == 64) return launch_write_ring_d<64>(ea, run, st);
  return launch_write_ring_d<128>(ea, run, st);
}
template <int DP>
int launch_pack_ring_d(const PrepArgs &pa, const RingRun &run, cudaStream_t st) {
  const size_t smem = ring_pack_smem<DP>();
  if (cudaFuncSetAttribute(packtc_ring_kernel<DP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return RA_ERR_CUDA;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  packtc_ring_kernel<DP><<<(unsigned)(sms > 0 ? 2 * sms : 2), kRingThreads, smem, st>>>(
      pa, run);
  return RA_OK;
}
int launch_pack_ring(int DP, const PrepArgs &pa, const RingRun &run, cudaStream_t st) {
  if (DP == 32) return launch_pack_ring_d<32>(pa, run, st);
  if (DP == 64) return launch_pack_ring_d<64>(pa, run, st);
  return launch_pack_ring_d<128>(pa, run, st);
}
int launch_statsw_ring(int DP, const PrepArgs &pa, const RingRun &run, cudaStream_t st) {
  if (DP == 32) return launch_statsw_ring_d<32>(pa, run, st);
  if (DP == 64) return launch_statsw_ring_d<64>(pa, run, st);
  return launch_statsw_ring_d<128>(pa, run, st);
}

unsigned chunk_grid(const Layout &L) {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms < 1) sms = 1;
  const int64_t g = (int64_t)sms * kChunkCtasPerSm;
  return (unsigned)(L.max_chunks < g ? L.max_chunks : g);
}

// The rows-only instantiations of the deterministic mode (a gradient mode:
// without one the default kernel has no column sums and no atomics anyway).
int launch_tiles3_rows(int mode, const Tiles3Args &Targs, cudaStream_t st, int sms) {
  int per_sm = 0;
  cudaError_t e = mode == 2
      ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tiles3_kernel<2, true>, kT3Threads, 0)
      : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tiles3_kernel<1, true>, kT3Threads,
                                                      0);
  if (e != cudaSuccess) return RA_ERR_CUDA;
  if (per_sm < 1) per_sm = 1;
  if (mode == 2)
    tiles3_kernel<2, true><<<sms * per_sm, kT3Threads, 0, st>>>(Targs);
  else
    tiles3_kernel<1, true><<<sms * per_sm, kT3Threads, 0, st>>>(Targs);
  ++g_launches;
  return cuda_status(cudaGetLastError());
}

int launch_tiles3(int mode, bool rows, const Tiles3Args &Targs, cudaStream_t st) {
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (rows && mode != 0) return launch_tiles3_rows(mode, Targs, st, sms);
  cudaError_t e;
  constexpr int T = kT3Threads;
  if (mode == 0)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tiles3_kernel<0>, T, 0);
  else if (mode == 1)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tiles3_kernel<1>, T, 0);
  else if (mode == 2)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tiles3_kernel<2>, T, 0);
  else
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tiles3_kernel<3>, T, 0);
  if (e != cudaSuccess) return RA_ERR_CUDA;
  if (per_sm < 1) per_sm = 1;
  const int grid = sms * per_sm;
  if (mode == 0)
    tiles3_kernel<0><<<grid, kT3Threads, 0, st>>>(Targs);
  else if (mode == 1)
    tiles3_kernel<1><<<grid, kT3Threads, 0, st>>>(Targs);
  else if (mode == 2)
    tiles3_kernel<2><<<grid, kT3Threads, 0, st>>>(Targs);
  else
    tiles3_kernel<3><<<grid, kT3Threads, 0, st>>>(Targs);
  ++g_launches;
  return cuda_status(cudaGetLastError());
}

template <int DP>
void launch_tilesg_dp(int mode, int64_t grid, const TilesGArgs &T, cudaStream_t st) {
  if (mode == 0)
    tilesg_kernel<DP, 0><<<(unsigned)grid, kGenRows, 0, st>>>(T);
  else if (mode == 1)
    tilesg_kernel<DP, 1><<<(unsigned)grid, kGenRows, 0, st>>>(T);
  else  // mode 2: sigma gradient
    tilesg_kernel<DP, 2><<<(unsigned)grid, kGenRows, 0, st>>>(T);
}

template <int DP, int MODE>
int launch_tc16_dm(int64_t max_items, const Tc16Args &T, cudaStream_t st) {
  const size_t smem = t16_smem_request(DP);
  static_assert(t16_smem_bytes(DP) <= t16_smem_request(DP), "shared memory request too small");
  if (cudaFuncSetAttribute(tilestc16_kernel<DP, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return RA_ERR_CUDA;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t grid = sms > 0 ? sms : 1;  // one persistent CTA per SM
  if (grid > max_items) grid = max_items;
  tilestc16_kernel<DP, MODE><<<(unsigned)grid, kT16Threads, smem, st>>>(T);
  return cuda_status(cudaGetLastError());
}

template <int DP>
int launch_tc16_d(int mode, int64_t max_items, const Tc16Args &T, cudaStream_t st) {
  if (mode == 0) return launch_tc16_dm<DP, 0>(max_items, T, st);
  if (mode == 1) return launch_tc16_dm<DP, 1>(max_items, T, st);
  return launch_tc16_dm<DP, 2>(max_items, T, st);  // mode 2: sigma gradient
}

int launch_tc16(int DP, int mode, int64_t max_items, const Tc16Args &T, cudaStream_t st) {
  int rc;
  switch (DP) {
    case 32: rc = launch_tc16_d<32>(mode, max_items, T, st); break;
    case 64: rc = launch_tc16_d<64>(mode, max_items, T, st); break;
    case 128: rc = launch_tc16_d<128>(mode, max_items, T, st); break;
    default: return RA_ERR_INVALID_ARGUMENT;
  }
  ++g_launches;
  return rc;
}

int launch_tilesg(int DP, int mode, int64_t grid, const TilesGArgs &T, cudaStream_t st) {
  switch (DP) {
    case 4: launch_tilesg_dp<4>(mode, grid, T, st); break;
    case 8: launch_tilesg_dp<8>(mode, grid, T, st); break;
    case 16: launch_tilesg_dp<16>(mode, grid, T, st); break;
    case 32: launch_tilesg_dp<32>(mode, grid, T, st); break;
    case 64: launch_tilesg_dp<64>(mode, grid, T, st); break;
    case 128: launch_tilesg_dp<128>(mode, grid, T, st); break;
    case 256: launch_tilesg_dp<256>(mode, grid, T, st); break;
    default: return RA_ERR_INVALID_ARGUMENT;
  }
  ++g_launches;
  return cuda_status(cudaGetLastError());
}

int finish_impl(const ra_kde_desc *d, const Layout &L, double *Kxx, double *Kyy, double *Kxy,
                void *ws, cudaStream_t st);

// D <= 3 in the deterministic mode with gradients: both orientations, rows
// only (tiles3_kernel<MODE, true>).
bool rows_only(const ra_kde_desc *d) {
  return d->dim <= 3 && d->deterministic && d->need_grad;
}

// Whether a pair may have more than kSmallPts points on a side (the D <= 3
// layout's chunked passes are launched only then; they skip small pairs).
bool may_have_large_pairs(const ra_kde_desc *d) {
  return d->layout == RA_LAYOUT_DENSE ? (d->nmax_x > kSmallPts || d->nmax_y > kSmallPts)
                                      : (d->num_x > kSmallPts || d->num_y > kSmallPts);
}

int check_inputs(const ra_kde_desc *d, const ra_kde_inputs *in) {
  if (in == nullptr) return RA_ERR_INVALID_ARGUMENT;
  if ((d->num_x > 0 && in->x == nullptr) || (d->num_y > 0 && in->y == nullptr))
    return RA_ERR_INVALID_ARGUMENT;
  if (d->layout == RA_LAYOUT_RAGGED && d->num_pairs > 0 &&
      (in->ptr_x == nullptr || in->ptr_y == nullptr))
    return RA_ERR_INVALID_ARGUMENT;
  return RA_OK;
}

// Forward, first phase: everything up to the tile kernels (segments, ptr
// checks, sums, metadata, work plan, packing).  Every data error the forward
// can find in its inputs is in the workspace's error word when it is done.
int prepare_impl(const ra_kde_desc *d, const ra_kde_inputs *in, void *ws, size_t ws_bytes,
                 cudaStream_t st) {
  const Layout L = make_layout(d);
  int rc = check_common(d, ws, ws_bytes, L.total);
  if (rc) return rc;
  rc = check_inputs(d, in);
  if (rc) return rc;
  const int64_t P = d->num_pairs;
  // header: error word, ticket, state flag, item count
  if (cudaMemsetAsync(ws, 0, kHdrBytes, st) != cudaSuccess) return RA_ERR_CUDA;
  if (P == 0) return RA_OK;
  const bool grad = d->need_grad != 0;
  const int mode = !grad ? 0 : (d->need_sigma_grad ? 2 : (d->skip_weight_sums ? 3 : 1));
  // the per-point sums start at zero where kernels add into them (the D <= 3
  // tile kernel's column sums) or where a split evaluation sums the records
  // of all shards.  The tensor-core kernel writes every field of every valid
  // row itself (an item exists for each orientation and row tile, zeros when
  // it has no column tiles), so there a clear would only cost bandwidth (0.6
  // GB per step for 1024 graphs at D=128); in the D <= 3 layout the packing
  // clears each slot it packs (prep3_kernel, pack3_kernel), stores that a
  // latency-bound kernel absorbs, instead of a separate pass.
  const bool acc_written = (L.tc16 || L.packed3) && !(d->shard_count > 1);
  if (grad && !acc_written) {
    if (cudaMemsetAsync(at<char>(ws, L.accX), 0, L.acc_x_bytes, st) != cudaSuccess ||
        cudaMemsetAsync(at<char>(ws, L.accY), 0, L.acc_y_bytes, st) != cudaSuccess)
      return RA_ERR_CUDA;
  }
  const float scale = scale_for(d->sigma);

  // ---- prep ----
  PrepArgs pa;
  std::memset(&pa, 0, sizeof(pa));
  pa.P = P;
  pa.D = d->dim;
  pa.DP = L.DP;
  pa.layout = d->layout;
  pa.wmode_x = d->weights_x;
  pa.wmode_y = d->weights_y;
  pa.center = d->center;
  pa.num_x = d->num_x;
  pa.num_y = d->num_y;
  pa.nmax_x = d->nmax_x;
  pa.nmax_y = d->nmax_y;
  pa.chunk_cap = L.max_chunks;
  pa.scale = scale;
  pa.sigma_p = in->sigma_pairs;
  pa.x = in->x;
  pa.y = in->y;
  pa.w_x = in->w_x;
  pa.w_y = in->w_y;
  pa.ptr_x = in->ptr_x;
  pa.ptr_y = in->ptr_y;
  pa.mask_x = d->layout == RA_LAYOUT_DENSE ? in->mask_x : nullptr;
  pa.mask_y = d->layout == RA_LAYOUT_DENSE ? in->mask_y : nullptr;
  pa.seg = at<Seg>(ws, L.seg);
  pa.meta = at<double>(ws, L.meta);
  pa.rec = at<double>(ws, L.rec);
  pa.chcnt = at<int64_t>(ws, L.chcnt);
  pa.chx = at<int64_t>(ws, L.chx);
  pa.choff = at<int64_t>(ws, L.choff);
  pa.cpair = at<int32_t>(ws, L.cpair);
  pa.ticket = at<unsigned>(ws, L.hdr + kHdrChunkTickets);  // the sums pass
  pa.pair_ticket = at<unsigned>(ws, L.hdr + kHdrChunkTickets) + 4;
  pa.err = at<int>(ws, L.hdr + kHdrErr);
  pa.allow_fold = mode == 2 ? 0 : 1;
  if (!L.packed3) {
    pa.Gx = at<float>(ws, L.Gx);
    pa.Gy = at<float>(ws, L.Gy);
    pa.Ax = at<float>(ws, L.Ax);
    pa.Ay = at<float>(ws, L.Ay);
  }
  if (L.tc16) {
    pa.tc16 = 1;
    pa.tcnt = at<int64_t>(ws, L.cnt) + P;  // free until the plan counts items
    pa.tbase_x = at<int64_t>(ws, L.tbase_x);
    pa.tbase_y = at<int64_t>(ws, L.tbase_y);
    pa.hx = at<uint8_t>(ws, L.hx);
    pa.hy = at<uint8_t>(ws, L.hy);
    pa.lx = at<uint8_t>(ws, L.lx);
    pa.ly = at<uint8_t>(ws, L.ly);
    pa.cx = at<float>(ws, L.cx);
    pa.cy = at<float>(ws, L.cy);
  }
  PackArgs pk;
  std::memset(&pk, 0, sizeof(pk));
  if (L.packed3) {
    pa.tcnt = at<int64_t>(ws, L.cnt) + P;  // free until the plan counts items
    pa.tbase_x = at<int64_t>(ws, L.tbase_x);
    pa.tbase_y = at<int64_t>(ws, L.tbase_y);
    pk.P = P;
    pk.D = d->dim;
    pk.nq = L.nq;
    pk.scale = scale;
    pk.sigma_p = in->sigma_pairs;
    pk.x = in->x;
    pk.y = in->y;
    pk.w_x = in->w_x;
    pk.w_y = in->w_y;
    pk.mask_x = pa.mask_x;
    pk.mask_y = pa.mask_y;
    pk.wmode_x = d->weights_x;
    pk.wmode_y = d->weights_y;
    pk.seg = at<Seg>(ws, L.seg);
    pk.meta = at<double>(ws, L.meta);
    pk.choff = at<int64_t>(ws, L.choff);
    pk.chx = at<int64_t>(ws, L.chx);
    pk.cpair = at<int32_t>(ws, L.cpair);
    pk.ticket = at<unsigned>(ws, L.hdr + kHdrChunkTickets) + 1;  // packing
    pk.tbase_x = at<int64_t>(ws, L.tbase_x);
    pk.tbase_y = at<int64_t>(ws, L.tbase_y);
    pk.max_tiles_x = L.max_tiles_x;
    pk.max_tiles_y = L.max_tiles_y;
    pk.tiles_x = at<ulonglong2>(ws, L.tiles_x);
    pk.tiles_y = at<ulonglong2>(ws, L.tiles_y);
    pk.aw_x = at<float>(ws, L.Ax);
    pk.aw_y = at<float>(ws, L.Ay);
    if (grad && !(d->shard_count > 1)) {  // cleared with the packing (below)
      pk.acc_x = at<float>(ws, L.accX);
      pk.acc_y = at<float>(ws, L.accY);
    }
  }
  const unsigned cgrid = chunk_grid(L);
  segment_kernel<<<1, 1024, 0, st>>>(pa);
  ++g_launches;
  // D <= 3: pairs with at most kSmallPts points per side are prepared by one
  // CTA each (sums, metadata, packing); the chunked passes below take the rest
  // and are launched only when a pair can be larger
  const bool may_be_large = may_have_large_pairs(d);
  if (L.packed3) {
    prep3_kernel<kPrepThreads>
        <<<(unsigned)(P < (int64_t)cgrid ? P : (int64_t)cgrid), kPrepThreads, 0, st>>>(pa, pk);
    ++g_launches;
    if (may_be_large) {
      stats3_kernel<kPrepThreads><<<cgrid, kPrepThreads, 0, st>>>(pa);
      meta_kernel<<<(unsigned)ceil_div(P, 4), 128, 0, st>>>(pa);
      g_launches += 2;
    }
  } else {
    // float4 loads of the caller's points need D % 4 == 0 and 16-byte
    // aligned bases; anything else takes the scalar passes
    const bool v4 = d->dim % 4 == 0 && aligned16(in->x) && aligned16(in->y);
    // equal weights and no mask: the rows are the points alone, streamed by
    // bulk copies (ra_ring.cuh)
    const bool ring = v4 && L.DP >= 32 && L.DP <= 128 && pa.mask_x == nullptr && pa.mask_y == nullptr &&
                      (d->weights_x == RA_WEIGHTS_UNIFORM || in->w_x == nullptr) &&
                      (d->weights_y == RA_WEIGHTS_UNIFORM || in->w_y == nullptr);
    if (ring) {
      const int rg = launch_statsw_ring(L.DP, pa, ring_run(d), st);
      if (rg) return rg;
    } else if (v4 && L.DP == 32)
      statsw4_kernel<32><<<cgrid, 256, 0, st>>>(pa);
    else if (v4 && L.DP == 64)
      statsw4_kernel<64><<<cgrid, 256, 0, st>>>(pa);
    else if (v4 && L.DP == 128)
      statsw4_kernel<128><<<cgrid, 256, 0, st>>>(pa);
    else if (v4 && L.DP == 256)
      statsw4_kernel<256><<<cgrid, 256, 0, st>>>(pa);
    else if (L.DP == 32)
      statsw_kernel<32><<<cgrid, 256, 0, st>>>(pa);
    else if (L.DP == 64)
      statsw_kernel<64><<<cgrid, 256, 0, st>>>(pa);
    else if (L.DP == 128)
      statsw_kernel<128><<<cgrid, 256, 0, st>>>(pa);
    else if (L.DP == 256)
      statsw_kernel<256><<<cgrid, 256, 0, st>>>(pa);
    else
      stats_kernel<kPrepThreads><<<cgrid, kPrepThreads, 0, st>>>(pa);
    meta_kernel<<<(unsigned)ceil_div(P, 4), 128, 0, st>>>(pa);
    pa.ticket = at<unsigned>(ws, L.hdr + kHdrChunkTickets) + 1;  // packing
    if (L.tc16 && ring) {
      const int rg = launch_pack_ring(L.DP, pa, ring_run(d), st);
      if (rg) return rg;
    } else if (L.tc16 && v4 && L.DP == 32)
      packtc_kernel<32, true><<<cgrid, 256, 0, st>>>(pa);
    else if (L.tc16 && v4 && L.DP == 64)
      packtc_kernel<64, true><<<cgrid, 256, 0, st>>>(pa);
    else if (L.tc16 && v4 && L.DP == 128)
      packtc_kernel<128, true><<<cgrid, 256, 0, st>>>(pa);
    else if (L.tc16 && L.DP == 32)
      packtc_kernel<32, false><<<cgrid, 256, 0, st>>>(pa);
    else if (L.tc16 && L.DP == 64)
      packtc_kernel<64, false><<<cgrid, 256, 0, st>>>(pa);
    else if (L.tc16 && L.DP == 128)
      packtc_kernel<128, false><<<cgrid, 256, 0, st>>>(pa);
    else if (v4 && L.DP == 32)
      packgw_kernel<32><<<cgrid, 256, 0, st>>>(pa);
    else if (v4 && L.DP == 64)
      packgw_kernel<64><<<cgrid, 256, 0, st>>>(pa);
    else if (v4 && L.DP == 128)
      packgw_kernel<128><<<cgrid, 256, 0, st>>>(pa);
    else if (v4 && L.DP == 256)
      packgw_kernel<256><<<cgrid, 256, 0, st>>>(pa);
    else
      packg_kernel<kPrepThreads><<<cgrid, kPrepThreads, 0, st>>>(pa);
    g_launches += 3;
  }
  if (cudaGetLastError() != cudaSuccess) return RA_ERR_CUDA;

  // ---- plan ----
  PlanArgs pl;
  pl.P = P;
  pl.generic = L.packed3 ? (rows_only(d) ? 2 : 0) : 1;
  pl.seg = at<Seg>(ws, L.seg);
  pl.cnt = at<int64_t>(ws, L.cnt);
  pl.boff = at<int64_t>(ws, L.boff);
  pl.item_off = at<int64_t>(ws, L.item_off);
  pl.n_items = at<int64_t>(ws, L.hdr + kHdrNItems);
  pl.items = at<Item>(ws, L.items);
  pl.max_items = L.max_items;
  pl.order = L.packed3 ? at<int32_t>(ws, L.order) : nullptr;
  pl.hist = L.packed3 ? at<int32_t>(ws, L.hdr + kHdrSizeHist) : nullptr;
  pl.cursor = L.packed3 ? pl.hist + kSizeBuckets : nullptr;
  pl.bbase = L.packed3 ? pl.hist + 2 * kSizeBuckets : nullptr;
  plan_count_kernel<<<(unsigned)ceil_div(P, 256), 256, 0, st>>>(pl);
  plan_scan_kernel<<<1, 1024, 0, st>>>(pl);
  plan_emit_kernel<<<(unsigned)P, 256, 0, st>>>(pl);
  g_launches += 3;
  if (cudaGetLastError() != cudaSuccess) return RA_ERR_CUDA;

  // ---- the tensor-core path's per-item records (the plan is complete) ----
  if (L.tc16) {
    const Seg *sg = at<Seg>(ws, L.seg);
    const double *mt = at<double>(ws, L.meta);
    const int64_t *tbx = at<int64_t>(ws, L.tbase_x), *tby = at<int64_t>(ws, L.tbase_y);
    const Item *itm = at<Item>(ws, L.items);
    const int64_t *nit = at<int64_t>(ws, L.hdr + kHdrNItems);
    ItemX *ixp = at<ItemX>(ws, L.ix);
    const unsigned ig = (unsigned)(L.max_items < 256 * 1184 ? ceil_div(L.max_items, (int64_t)256)
                                                            : 1184);
    if (L.DP == 32)
      t16_items_kernel<32><<<ig, 256, 0, st>>>(itm, nit, sg, mt, tbx, tby, ixp);
    else if (L.DP == 64)
      t16_items_kernel<64><<<ig, 256, 0, st>>>(itm, nit, sg, mt, tbx, tby, ixp);
    else
      t16_items_kernel<128><<<ig, 256, 0, st>>>(itm, nit, sg, mt, tbx, tby, ixp);
    ++g_launches;
    if (cudaGetLastError() != cudaSuccess) return RA_ERR_CUDA;
  }

  // ---- pack the large pairs' D <= 3 tiles (their metadata is complete) ----
  if (L.packed3 && may_be_large) {
    pack3_kernel<kPrepThreads><<<cgrid, kPrepThreads, 0, st>>>(pk);
    ++g_launches;
    if (cudaGetLastError() != cudaSuccess) return RA_ERR_CUDA;
  }
  return RA_OK;
}

// Forward, second phase: the tile kernels and (unless the problem is split
// over shards) the per-pair K.  Follows prepare_impl on the same stream.
int compute_impl(const ra_kde_desc *d, const ra_kde_inputs *in, double *Kxx, double *Kyy,
                 double *Kxy, void *ws, size_t ws_bytes, cudaStream_t st, cudaEvent_t ev0,
                 cudaEvent_t ev1) {
  const Layout L = make_layout(d);
  int rc = check_common(d, ws, ws_bytes, L.total);
  if (rc) return rc;
  rc = check_inputs(d, in);
  if (rc) return rc;
  if (Kxx == nullptr || Kyy == nullptr || Kxy == nullptr) return RA_ERR_INVALID_ARGUMENT;
  const int64_t P = d->num_pairs;
  if (P == 0) return RA_OK;
  const bool grad = d->need_grad != 0;
  const int mode = !grad ? 0 : (d->need_sigma_grad ? 2 : (d->skip_weight_sums ? 3 : 1));

  const bool sharded = d->shard_count > 1;
  const int sh_idx = sharded ? d->shard_index : 0, sh_cnt = sharded ? d->shard_count : 1;
  if (sharded && cudaMemsetAsync(at<char>(ws, L.itemK), 0,
                                 sizeof(double) * kItemF64 * (size_t)L.max_items,
                                 st) != cudaSuccess)
    return RA_ERR_CUDA;  // items of other shards contribute zeros to the reduction

  // ---- tiles ----
  if (ev0 != nullptr && cudaEventRecord(ev0, st) != cudaSuccess) return RA_ERR_CUDA;
  if (L.packed3) {
    Tiles3Args T;
    T.items = at<Item>(ws, L.items);
    T.n_items = at<int64_t>(ws, L.hdr + kHdrNItems);
    T.ticket = at<unsigned>(ws, L.hdr + kHdrTicket);
    T.seg = at<Seg>(ws, L.seg);
    T.tbase_x = at<int64_t>(ws, L.tbase_x);
    T.tbase_y = at<int64_t>(ws, L.tbase_y);
    T.tiles_x = at<ulonglong2>(ws, L.tiles_x);
    T.tiles_y = at<ulonglong2>(ws, L.tiles_y);
    T.aw_x = at<float>(ws, L.Ax);
    T.aw_y = at<float>(ws, L.Ay);
    T.meta = at<double>(ws, L.meta);
    T.acc_x = grad ? at<float>(ws, L.accX) : nullptr;
    T.acc_y = grad ? at<float>(ws, L.accY) : nullptr;
    T.itemK = at<double>(ws, L.itemK);
    T.itemS = at<double>(ws, L.itemS);
    T.shard_index = sh_idx;
    T.shard_count = sh_cnt;
    // largest items first; a split evaluation keeps the plan order, which
    // every shard derives alike (the sorted order within a cost is not)
    T.order = sharded ? nullptr : at<int32_t>(ws, L.order);
    rc = launch_tiles3(mode, rows_only(d), T, st);
    if (rc) return rc;
  } else {
    TilesGArgs T;
    T.items = at<Item>(ws, L.items);
    T.n_items = at<int64_t>(ws, L.hdr + kHdrNItems);
    T.seg = at<Seg>(ws, L.seg);
    T.Gx = at<float>(ws, L.Gx);
    T.Gy = at<float>(ws, L.Gy);
    T.Ax = at<float>(ws, L.Ax);
    T.Ay = at<float>(ws, L.Ay);
    T.accX = grad ? at<float>(ws, L.accX) : nullptr;
    T.accY = grad ? at<float>(ws, L.accY) : nullptr;
    T.itemK = at<double>(ws, L.itemK);
    T.itemS = at<double>(ws, L.itemS);
    T.need_rows = grad ? 1 : 0;
    T.shard_index = sh_idx;
    T.shard_count = sh_cnt;
    T.err = at<int>(ws, L.hdr + kHdrErr);
    T.no_mma = (d->test_hooks & RA_TEST_NO_MMA) ? 1 : 0;
    T.spin_limit = T.no_mma ? 4096u : kTcSpinLimit;
    // the generic kernels keep every per-point sum anyway: mode 3 (no column
    // weight sums, a D <= 3 distinction) is their mode 1
    const int gmode = mode == 3 ? 1 : mode;
    if (L.tc16) {
      Tc16Args C;
      std::memset(&C, 0, sizeof(C));
      C.items = T.items;
      C.ix = at<ItemX>(ws, L.ix);
      C.n_items = T.n_items;
      C.seg = T.seg;
      C.meta = at<double>(ws, L.meta);
      C.tbase_x = at<int64_t>(ws, L.tbase_x);
      C.tbase_y = at<int64_t>(ws, L.tbase_y);
      C.hx = at<uint8_t>(ws, L.hx);
      C.hy = at<uint8_t>(ws, L.hy);
      C.lx = at<uint8_t>(ws, L.lx);
      C.ly = at<uint8_t>(ws, L.ly);
      C.cx = at<float>(ws, L.cx);
      C.cy = at<float>(ws, L.cy);
      C.Ax = T.Ax;
      C.Ay = T.Ay;
      C.accX = T.accX;
      C.accY = T.accY;
      C.itemK = T.itemK;
      C.itemS = T.itemS;
      C.need_rows = T.need_rows;
      C.shard_index = T.shard_index;
      C.shard_count = T.shard_count;
      C.err = T.err;
      C.spin_limit = T.spin_limit;
      C.no_mma = T.no_mma;
      rc = launch_tc16(L.DP, gmode, L.max_items, C, st);
    } else {
      rc = launch_tilesg(L.DP, gmode, L.max_items, T, st);
    }
    if (rc) return rc;
  }

  if (ev1 != nullptr && cudaEventRecord(ev1, st) != cudaSuccess) return RA_ERR_CUDA;
  if (sharded) return RA_OK;  // partials are reduced by the caller, then finish_impl
  return finish_impl(d, L, Kxx, Kyy, Kxy, ws, st);
}

int forward_impl(const ra_kde_desc *d, const ra_kde_inputs *in, double *Kxx, double *Kyy,
                 double *Kxy, void *ws, size_t ws_bytes, cudaStream_t st,
                 cudaEvent_t ev0 = nullptr, cudaEvent_t ev1 = nullptr) {
  if (Kxx == nullptr || Kyy == nullptr || Kxy == nullptr) return RA_ERR_INVALID_ARGUMENT;
  const int rc = prepare_impl(d, in, ws, ws_bytes, st);
  if (rc) return rc;
  return compute_impl(d, in, Kxx, Kyy, Kxy, ws, ws_bytes, st, ev0, ev1);
}

// Per-pair K from the item partials (into the caller's arrays), the state flag.
int finish_impl(const ra_kde_desc *d, const Layout &L, double *Kxx, double *Kyy, double *Kxy,
                void *ws, cudaStream_t st) {
  const int64_t P = d->num_pairs;
  const bool grad = d->need_grad != 0;
  if (P == 0) return RA_OK;
  // ---- finalize ----
  FinalizeArgs fa;
  fa.P = P;
  fa.item_off = at<int64_t>(ws, L.item_off);
  fa.boff = at<int64_t>(ws, L.boff);
  fa.itemK = at<double>(ws, L.itemK);
  fa.itemS = at<double>(ws, L.itemS);
  fa.K_ws = at<double>(ws, L.Kws);
  fa.S_ws = at<double>(ws, L.Sws);
  // the caller's three K arrays are written by the kernel itself
  fa.K_out[0] = Kxx;
  fa.K_out[1] = Kyy;
  fa.K_out[2] = Kxy;
  // the state flag marks a workspace whose forward kept what a backward needs;
  // the kernel writes it, so no host memory is involved
  fa.state = grad ? at<int>(ws, L.hdr + kHdrState) : nullptr;
  finalize_warp_kernel<<<(unsigned)ceil_div(P, 8), 256, 0, st>>>(fa);
  ++g_launches;
  // pairs of at most kSmallPts points per side have at most 192 items
  static_assert(kWarpItems >= 3 * (kSmallPts / kTile), "small pairs fit one warp");
  if (may_have_large_pairs(d)) {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t g = (int64_t)(sms > 0 ? sms : 1) * 4;  // a stride over the pairs
    finalize_kernel<256><<<(unsigned)(P < g ? P : g), 256, 0, st>>>(fa);
    ++g_launches;
  }
  return cuda_status(cudaGetLastError());
}

int backward_impl(const ra_kde_desc *d, const ra_kde_inputs *in, const double *coef,
                  const ra_kde_grads *gr, void *ws, size_t ws_bytes, cudaStream_t st) {
  const Layout L = make_layout(d);
  int rc = check_common(d, ws, ws_bytes, L.total);
  if (rc) return rc;
  if (in == nullptr || gr == nullptr || coef == nullptr) return RA_ERR_INVALID_ARGUMENT;
  if (!d->need_grad) return RA_ERR_STATE;
  if (gr->grad_sigma != nullptr && !d->need_sigma_grad) return RA_ERR_STATE;
  if (d->skip_weight_sums && (gr->grad_wx != nullptr || gr->grad_wy != nullptr))
    return RA_ERR_STATE;
  const int64_t P = d->num_pairs;
  if (P == 0) return RA_OK;
  EpilogueArgs ea;
  std::memset(&ea, 0, sizeof(ea));
  ea.P = P;
  ea.D = d->dim;
  ea.DP = L.DP;
  ea.packed3 = L.packed3 ? 1 : 0;
  ea.center = d->center;
  ea.wmode_x = d->weights_x;
  ea.wmode_y = d->weights_y;
  ea.scale = (double)scale_for(d->sigma);
  ea.sigma = d->sigma;
  ea.sigma_p = in->sigma_pairs;
  ea.seg = at<Seg>(ws, L.seg);
  ea.meta = at<double>(ws, L.meta);
  ea.coef = coef;
  ea.S_ws = at<double>(ws, L.Sws);
  ea.choff = at<int64_t>(ws, L.choff);
  ea.chx = at<int64_t>(ws, L.chx);
  ea.cpair = at<int32_t>(ws, L.cpair);
  // the chunked passes' and epi3_small_kernel's tickets, zeroed here: a
  // backward may run more than once after its forward
  unsigned *const etk = at<unsigned>(ws, L.hdr + kHdrChunkTickets) + 2;
  if (cudaMemsetAsync(etk, 0, 4 * sizeof(unsigned), st) != cudaSuccess) return RA_ERR_CUDA;
  ea.pair_ticket = etk + 3;
  ea.rec = at<double>(ws, L.rec);
  ea.x = in->x;
  ea.y = in->y;
  ea.mask_x = d->layout == RA_LAYOUT_DENSE ? in->mask_x : nullptr;
  ea.mask_y = d->layout == RA_LAYOUT_DENSE ? in->mask_y : nullptr;
  if (L.packed3) {
    ea.tiles_x = at<ulonglong2>(ws, L.tiles_x);
    ea.tiles_y = at<ulonglong2>(ws, L.tiles_y);
    ea.tbase_x = at<int64_t>(ws, L.tbase_x);
    ea.tbase_y = at<int64_t>(ws, L.tbase_y);
    ea.nq = L.nq;
    ea.aw_x = at<float>(ws, L.Ax);
    ea.aw_y = at<float>(ws, L.Ay);
  } else {
    ea.Gx = at<float>(ws, L.Gx);
    ea.Gy = at<float>(ws, L.Gy);
    ea.Ax = at<float>(ws, L.Ax);
    ea.Ay = at<float>(ws, L.Ay);
  }
  ea.accX = at<float>(ws, L.accX);
  ea.accY = at<float>(ws, L.accY);
  ea.acc_stride = L.acc_stride;
  ea.grad_x = gr->grad_x;
  ea.grad_y = gr->grad_y;
  ea.grad_wx = gr->grad_wx;
  ea.grad_wy = gr->grad_wy;
  ea.grad_sigma = gr->grad_sigma;
  ea.totals = d->center || (gr->grad_wx != nullptr && d->weights_x != RA_WEIGHTS_UNIFORM) ||
              (gr->grad_wy != nullptr && d->weights_y != RA_WEIGHTS_UNIFORM);
  // tensor-core layout: no fp32 copy of the packed coordinates; the backward
  // packs them again from the points
  ea.xraw = L.tc16 ? 1 : 0;
  ea.vec4 = d->dim % 4 == 0 && aligned16(gr->grad_x) && aligned16(gr->grad_y) &&
            (!ea.xraw || (aligned16(in->x) && aligned16(in->y)));
  const unsigned cgrid = chunk_grid(L);
  if (L.packed3) {
    // small pairs: one CTA per pair (both passes); large pairs: chunked passes
    epi3_small_kernel<kEpiThreads>
        <<<(unsigned)(P < (int64_t)cgrid ? P : (int64_t)cgrid), kEpiThreads, 0, st>>>(ea);
    ++g_launches;
    if (may_have_large_pairs(d)) {
      ea.ticket = etk;
      epi3_partial_kernel<kEpiThreads><<<cgrid, kEpiThreads, 0, st>>>(ea);
      ea.ticket = etk + 1;
      epi3_write_kernel<kEpiThreads><<<cgrid, kEpiThreads, 0, st>>>(ea);
      g_launches += 2;
    }
  } else if (L.DP >= 32 && L.DP <= 128 && ea.vec4 && ea.xraw && ea.mask_x == nullptr &&
             ea.mask_y == nullptr && ea.grad_wx == nullptr && ea.grad_wy == nullptr) {
    // tensor-core layout, position gradients only: the write pass streams its
    // rows by bulk copies (ra_ring.cuh); the partial pass (centring) as below
    ea.err = at<int>(ws, L.hdr + kHdrErr);
    ea.ticket = etk;
    if (ea.totals) {
      if (L.DP == 32) epigw_partial_kernel<32><<<cgrid, 256, 0, st>>>(ea);
      else if (L.DP == 64) epigw_partial_kernel<64><<<cgrid, 256, 0, st>>>(ea);
      else epigw_partial_kernel<128><<<cgrid, 256, 0, st>>>(ea);
    }
    ea.ticket = etk + 1;
    const int rg = launch_write_ring(L.DP, ea, ring_run(d), st);
    if (rg) return rg;
    g_launches += ea.totals ? 2 : 1;
  } else if (L.DP >= 32) {
    // the partial pass only makes the side totals R (centering) and Q (weight
    // gradients); an uncentred call without weight gradients skips it
    switch (L.DP) {
      case 32:
        ea.ticket = etk;
        if (ea.totals) epigw_partial_kernel<32><<<cgrid, 256, 0, st>>>(ea);
        ea.ticket = etk + 1;
        epigw_write_kernel<32><<<cgrid, 256, 0, st>>>(ea);
        break;
      case 64:
        ea.ticket = etk;
        if (ea.totals) epigw_partial_kernel<64><<<cgrid, 256, 0, st>>>(ea);
        ea.ticket = etk + 1;
        epigw_write_kernel<64><<<cgrid, 256, 0, st>>>(ea);
        break;
      case 128:
        ea.ticket = etk;
        if (ea.totals) epigw_partial_kernel<128><<<cgrid, 256, 0, st>>>(ea);
        ea.ticket = etk + 1;
        epigw_write_kernel<128><<<cgrid, 256, 0, st>>>(ea);
        break;
      default:
        ea.ticket = etk;
        if (ea.totals) epigw_partial_kernel<256><<<cgrid, 256, 0, st>>>(ea);
        ea.ticket = etk + 1;
        epigw_write_kernel<256><<<cgrid, 256, 0, st>>>(ea);
        break;
    }
    g_launches += ea.totals ? 2 : 1;
  } else {
    ea.ticket = etk;
    epig_partial_kernel<kEpiThreads><<<cgrid, kEpiThreads, 0, st>>>(ea);
    ea.ticket = etk + 1;
    epig_write_kernel<kEpiThreads><<<cgrid, kEpiThreads, 0, st>>>(ea);
    g_launches += 2;
  }
  if (ea.grad_sigma != nullptr) {
    sigma_grad_kernel<<<(unsigned)ceil_div(P, 256), 256, 0, st>>>(ea);
    ++g_launches;
  }
  return cuda_status(cudaGetLastError());
}

// coef = (g, g, -2 g) for the legacy MMD backward
__global__ void mmd_coef_kernel(int64_t P, const double *g, double *coef) {
  const int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (p >= P) return;
  const double v = g[p];
  coef[p] = v;
  coef[P + p] = v;
  coef[2 * P + p] = -2.0 * v;
}

ra_kde_desc legacy_desc(int layout, int64_t P, int64_t NX, int64_t NY, int64_t nmx, int64_t nmy,
                        int32_t D, double sigma, int grad) {
  ra_kde_desc d;
  std::memset(&d, 0, sizeof(d));
  d.num_pairs = P;
  d.dim = D;
  d.layout = layout;
  d.num_x = NX;
  d.num_y = NY;
  d.nmax_x = nmx;
  d.nmax_y = nmy;
  d.weights_x = RA_WEIGHTS_RAW;
  d.weights_y = RA_WEIGHTS_RAW;
  d.center = 0;
  d.need_grad = grad;
  d.need_sigma_grad = grad;
  d.sigma = sigma;
  return d;
}

// ---- FP32 peak probe -------------------------------------------------------
__global__ void fp32_probe_kernel(float *out, int iters, float seed) {
  f2_t acc[8];
  for (int i = 0; i < 8; ++i) acc[i] = pk(seed + threadIdx.x * 1e-3f + i, seed - i);
  const f2_t m = pk(0.9999f, 0.9999f), c = pk(1e-4f, 1e-4f);
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int u = 0; u < 16; ++u) {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fma2(acc[i], m, c);
    }
  }
  float s = 0.f;
  for (int i = 0; i < 8; ++i) s += lo_of(acc[i]) + hi_of(acc[i]);
  out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

// Fixed scratch of ra_kde_mmd_forward_segmented_noalloc.  In host code the
// name is only a stand-in: the device address comes from cudaGetSymbolAddress,
// looked up once per device with that device current.
constexpr size_t kNoallocScratchBytes = (size_t)64 << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

// The current device's address of the scratch array, looked up on every call
// (the lookup allocates nothing; the first one on a device may load the
// library's device code there, which is why that first call belongs before any
// stream capture).  Not cached, so a device reset leaves nothing stale.
int noalloc_scratch_address(void **out) {
  void *p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
    return RA_ERR_CUDA;
  *out = p;
  return RA_OK;
}

int status_of_error_word(int err) {
  if (err & kErrPtrStart) return RA_ERR_PTR_START;
  if (err & kErrPtrEnd) return RA_ERR_PTR_END;
  if (err & kErrPtrOrder) return RA_ERR_PTR_ORDER;
  if (err & kErrWeightSum) return RA_ERR_WEIGHT_SUM;
  if (err & kErrTimeout) return RA_ERR_DEVICE_TIMEOUT;
  if (err & kErrSigma) return RA_ERR_SIGMA;
  return RA_OK;
}

}  // namespace

// Loss and outputs of the P pairs from the float64 sums, and its derivative
// (ra_mmd_outputs, ra_mmd_outputs_backward).
namespace {
template <typename T>
__global__ void mmd_outputs_kernel(const double *K, int64_t P, int cosine, double eps, T *loss,
                                   T *kxx, T *kyy, T *kxy) {
  const int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (p >= P) return;
  const double a = K[p], b = K[P + p], c = K[2 * P + p];
  const double l = cosine ? 1.0 - c / sqrt(fmax(a * b, eps)) : a + b - 2.0 * c;
  loss[p] = (T)l;
  kxx[p] = (T)a;
  kyy[p] = (T)b;
  kxy[p] = (T)c;
}
template <typename T>
__device__ __forceinline__ double grad_at(const void *g, int64_t p) {
  return g == nullptr ? 0.0 : (double)static_cast<const T *>(g)[p];
}
template <typename T>
__global__ void mmd_outputs_backward_kernel(const double *K, int64_t P, int cosine, double eps,
                                            const void *gl, const void *ga, const void *gb,
                                            const void *gc, double *coef) {
  const int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (p >= P) return;
  const double gL = grad_at<T>(gl, p);
  double da, db, dc;  // dL/dKxx, dL/dKyy, dL/dKxy
  if (cosine) {
    const double a = K[p], b = K[P + p], c = K[2 * P + p];
    const double ab = a * b;
    const double s = sqrt(fmax(ab, eps));
    dc = -1.0 / s;
    // clamp_min passes its gradient where the product is not below eps
    const double ds = ab >= eps ? c / (2.0 * s * s * s) : 0.0;
    da = ds * b;
    db = ds * a;
  } else {
    da = 1.0;
    db = 1.0;
    dc = -2.0;
  }
  coef[p] = grad_at<T>(ga, p) + gL * da;
  coef[P + p] = grad_at<T>(gb, p) + gL * db;
  coef[2 * P + p] = grad_at<T>(gc, p) + gL * dc;
}
}  // namespace

extern "C" {

const char *ra_status_string(int status) {
  switch (status) {
    case RA_OK: return "ok";
    case RA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case RA_ERR_SIGMA: return "sigma must be positive";
    case RA_ERR_WORKSPACE: return "workspace too small or not 256-byte aligned";
    case RA_ERR_CUDA: return "CUDA error";
    case RA_ERR_PTR_START: return "ptr must start at 0";
    case RA_ERR_PTR_END: return "ptr[-1] must equal number of nodes";
    case RA_ERR_PTR_ORDER: return "ptr offsets must be non-decreasing";
    case RA_ERR_WEIGHT_SUM: return "weights must sum to a positive value per segment";
    case RA_ERR_STATE: return "backward needs a forward run with need_grad (and need_sigma_grad)";
    case RA_ERR_DEVICE_TIMEOUT:
      return "a bounded wait inside a kernel expired (tensor-core kernels or bulk-copy passes); "
             "results are invalid";
    case RA_ERR_SCRATCH_LIMIT:
      return "problem too large for the 64 MiB fixed scratch of the no-alloc entry point";
    default: return "unknown status";
  }
}

size_t ra_kde_workspace_bytes(const ra_kde_desc *desc) {
  if (!desc_ok(desc)) return 0;
  return make_layout(desc).total;
}

int ra_kde_forward(const ra_kde_desc *desc, const ra_kde_inputs *in, double *K, void *workspace,
                   size_t workspace_bytes, ra_stream_t stream) {
  if (!desc_ok(desc) || K == nullptr) return RA_ERR_INVALID_ARGUMENT;
  const int64_t P = desc->num_pairs;
  return forward_impl(desc, in, K, K + P, K + 2 * P, workspace, workspace_bytes,
                      (cudaStream_t)stream);
}

int ra_kde_forward_prepare(const ra_kde_desc *desc, const ra_kde_inputs *in, void *workspace,
                           size_t workspace_bytes, ra_stream_t stream) {
  if (!desc_ok(desc)) return RA_ERR_INVALID_ARGUMENT;
  return prepare_impl(desc, in, workspace, workspace_bytes, (cudaStream_t)stream);
}

int ra_kde_forward_compute(const ra_kde_desc *desc, const ra_kde_inputs *in, double *K,
                           void *workspace, size_t workspace_bytes, ra_stream_t stream) {
  if (!desc_ok(desc) || K == nullptr) return RA_ERR_INVALID_ARGUMENT;
  const int64_t P = desc->num_pairs;
  return compute_impl(desc, in, K, K + P, K + 2 * P, workspace, workspace_bytes,
                      (cudaStream_t)stream, nullptr, nullptr);
}

int ra_kde_backward(const ra_kde_desc *desc, const ra_kde_inputs *in, const double *coef,
                    const ra_kde_grads *grads, void *workspace, size_t workspace_bytes,
                    ra_stream_t stream) {
  return backward_impl(desc, in, coef, grads, workspace, workspace_bytes, (cudaStream_t)stream);
}

int ra_kde_forward_profiled(const ra_kde_desc *desc, const ra_kde_inputs *in, double *K,
                            void *workspace, size_t workspace_bytes, ra_stream_t stream,
                            float *tiles_ms) {
  if (!desc_ok(desc) || K == nullptr || tiles_ms == nullptr) return RA_ERR_INVALID_ARGUMENT;
  cudaEvent_t e0, e1;
  if (cudaEventCreate(&e0) != cudaSuccess) return RA_ERR_CUDA;
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return RA_ERR_CUDA;
  }
  const int64_t P = desc->num_pairs;
  int rc = forward_impl(desc, in, K, K + P, K + 2 * P, workspace, workspace_bytes,
                        (cudaStream_t)stream, e0, e1);
  *tiles_ms = 0.f;
  if (rc == RA_OK && P > 0) {
    if (cudaEventSynchronize(e1) != cudaSuccess || cudaEventElapsedTime(tiles_ms, e0, e1))
      rc = RA_ERR_CUDA;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return rc;
}

int ra_kde_partials(const ra_kde_desc *desc, void *workspace, size_t workspace_bytes,
                    double **f64_buf, size_t *f64_count, float **f32_buf, size_t *f32_count) {
  if (!desc_ok(desc) || f64_buf == nullptr || f64_count == nullptr || f32_buf == nullptr ||
      f32_count == nullptr)
    return RA_ERR_INVALID_ARGUMENT;
  const Layout L = make_layout(desc);
  if (workspace == nullptr || workspace_bytes < L.total) return RA_ERR_WORKSPACE;
  *f64_buf = at<double>(workspace, L.itemK);
  *f64_count = kItemF64 * (size_t)L.max_items;
  if (desc->need_grad) {
    *f32_buf = at<float>(workspace, L.accX);
    *f32_count = (L.accY + L.acc_y_bytes - L.accX) / sizeof(float);
  } else {
    *f32_buf = nullptr;
    *f32_count = 0;
  }
  return RA_OK;
}

int ra_kde_forward_finish(const ra_kde_desc *desc, double *K, void *workspace,
                          size_t workspace_bytes, ra_stream_t stream) {
  if (!desc_ok(desc) || K == nullptr) return RA_ERR_INVALID_ARGUMENT;
  const Layout L = make_layout(desc);
  const int rc = check_common(desc, workspace, workspace_bytes, L.total);
  if (rc) return rc;
  const int64_t P = desc->num_pairs;
  return finish_impl(desc, L, K, K + P, K + 2 * P, workspace, (cudaStream_t)stream);
}

int ra_kde_check(const void *workspace, ra_stream_t stream) {
  if (workspace == nullptr) return RA_ERR_INVALID_ARGUMENT;
  int err = 0;
  if (cudaMemcpyAsync(&err, static_cast<const char *>(workspace) + kHdrErr, sizeof(int),
                      cudaMemcpyDeviceToHost, (cudaStream_t)stream) != cudaSuccess)
    return RA_ERR_CUDA;
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return RA_ERR_CUDA;
  return status_of_error_word(err);
}

int ra_kde_status_of_error_word(int word) { return status_of_error_word(word); }

int ra_kde_error_word_async(const void *workspace, const int32_t *flags, int32_t nflags,
                            int32_t *host, ra_stream_t stream) {
  if (workspace == nullptr || host == nullptr || nflags < 0 || (nflags > 0 && flags == nullptr))
    return RA_ERR_INVALID_ARGUMENT;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemcpyAsync(host, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, st) !=
      cudaSuccess)
    return RA_ERR_CUDA;
  if (nflags > 0 && cudaMemcpyAsync(host + 1, flags, sizeof(int32_t) * (size_t)nflags,
                                    cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return RA_ERR_CUDA;
  return RA_OK;
}

int ra_mmd_outputs(const double *K, int64_t P, int cosine, double eps, int out_f64, void *loss,
                   void *Kxx, void *Kyy, void *Kxy, ra_stream_t stream) {
  if (P < 0 || (P > 0 && (K == nullptr || loss == nullptr || Kxx == nullptr || Kyy == nullptr ||
                          Kxy == nullptr)))
    return RA_ERR_INVALID_ARGUMENT;
  if (P == 0) return RA_OK;
  const unsigned grid = (unsigned)ceil_div(P, (int64_t)256);
  cudaStream_t st = (cudaStream_t)stream;
  if (out_f64)
    mmd_outputs_kernel<double><<<grid, 256, 0, st>>>(K, P, cosine, eps, (double *)loss,
                                                      (double *)Kxx, (double *)Kyy,
                                                      (double *)Kxy);
  else
    mmd_outputs_kernel<float><<<grid, 256, 0, st>>>(K, P, cosine, eps, (float *)loss,
                                                     (float *)Kxx, (float *)Kyy, (float *)Kxy);
  ++g_launches;
  return cuda_status(cudaGetLastError());
}

int ra_mmd_outputs_backward(const double *K, int64_t P, int cosine, double eps, int out_f64,
                            const void *g_loss, const void *g_Kxx, const void *g_Kyy,
                            const void *g_Kxy, double *coef, ra_stream_t stream) {
  if (P < 0 || (P > 0 && (K == nullptr || coef == nullptr))) return RA_ERR_INVALID_ARGUMENT;
  if (P == 0) return RA_OK;
  const unsigned grid = (unsigned)ceil_div(P, (int64_t)256);
  cudaStream_t st = (cudaStream_t)stream;
  if (out_f64)
    mmd_outputs_backward_kernel<double><<<grid, 256, 0, st>>>(K, P, cosine, eps, g_loss, g_Kxx,
                                                               g_Kyy, g_Kxy, coef);
  else
    mmd_outputs_backward_kernel<float><<<grid, 256, 0, st>>>(K, P, cosine, eps, g_loss, g_Kxx,
                                                              g_Kyy, g_Kxy, coef);
  ++g_launches;
  return cuda_status(cudaGetLastError());
}

size_t ra_kde_mmd_forward_workspace_bytes(int64_t B, int64_t Nx, int64_t Ny, int32_t D) {
  ra_kde_desc d = legacy_desc(RA_LAYOUT_DENSE, B, B * Nx, B * Ny, Nx, Ny, D, 1.0, 0);
  return ra_kde_workspace_bytes(&d);
}

int ra_kde_mmd_forward(const float *x, const float *y, const float *w_x, const float *w_y,
                       const uint8_t *mask_x, const uint8_t *mask_y, int64_t B, int64_t Nx,
                       int64_t Ny, int32_t D, double sigma, double *Kxx, double *Kyy,
                       double *Kxy, void *workspace, size_t workspace_bytes,
                       ra_stream_t stream) {
  if (B < 0 || Nx < 0 || Ny < 0) return RA_ERR_INVALID_ARGUMENT;
  if (B > 0 && (w_x == nullptr || w_y == nullptr || mask_x == nullptr || mask_y == nullptr))
    return RA_ERR_INVALID_ARGUMENT;
  ra_kde_desc d = legacy_desc(RA_LAYOUT_DENSE, B, B * Nx, B * Ny, Nx, Ny, D, sigma, 0);
  ra_kde_inputs in;
  std::memset(&in, 0, sizeof(in));
  in.x = x;
  in.y = y;
  in.w_x = w_x;
  in.w_y = w_y;
  in.mask_x = mask_x;
  in.mask_y = mask_y;
  return forward_impl(&d, &in, Kxx, Kyy, Kxy, workspace, workspace_bytes, (cudaStream_t)stream);
}

size_t ra_kde_mmd_forward_segmented_workspace_bytes(int64_t P, int64_t NX, int64_t NY,
                                                    int32_t D) {
  ra_kde_desc d = legacy_desc(RA_LAYOUT_RAGGED, P, NX, NY, 0, 0, D, 1.0, 0);
  return ra_kde_workspace_bytes(&d);
}

int ra_kde_mmd_forward_segmented(const float *x, const float *y, const float *w_x,
                                 const float *w_y, const int64_t *ptr_x, const int64_t *ptr_y,
                                 int64_t P, int64_t NX, int64_t NY, int32_t D, double sigma,
                                 double *Kxx, double *Kyy, double *Kxy, void *workspace,
                                 size_t workspace_bytes, ra_stream_t stream) {
  if ((NX > 0 && w_x == nullptr) || (NY > 0 && w_y == nullptr)) return RA_ERR_INVALID_ARGUMENT;
  ra_kde_desc d = legacy_desc(RA_LAYOUT_RAGGED, P, NX, NY, 0, 0, D, sigma, 0);
  ra_kde_inputs in;
  std::memset(&in, 0, sizeof(in));
  in.x = x;
  in.y = y;
  in.w_x = w_x;
  in.w_y = w_y;
  in.ptr_x = ptr_x;
  in.ptr_y = ptr_y;
  return forward_impl(&d, &in, Kxx, Kyy, Kxy, workspace, workspace_bytes, (cudaStream_t)stream);
}

size_t ra_kde_mmd_backward_segmented_workspace_bytes(int64_t P, int64_t NX, int64_t NY,
                                                     int32_t D) {
  ra_kde_desc d = legacy_desc(RA_LAYOUT_RAGGED, P, NX, NY, 0, 0, D, 1.0, 1);
  return ra_kde_workspace_bytes(&d);
}

int ra_kde_mmd_backward_segmented(const float *x, const float *y, const float *w_x,
                                  const float *w_y, const int64_t *ptr_x, const int64_t *ptr_y,
                                  int64_t P, int64_t NX, int64_t NY, int32_t D,
                                  const double *grad_loss, double sigma, float *grad_x,
                                  float *grad_y, double *grad_wx, double *grad_wy,
                                  double *grad_sigma_pairs, void *workspace,
                                  size_t workspace_bytes, ra_stream_t stream) {
  if ((NX > 0 && w_x == nullptr) || (NY > 0 && w_y == nullptr)) return RA_ERR_INVALID_ARGUMENT;
  if (P > 0 && grad_loss == nullptr) return RA_ERR_INVALID_ARGUMENT;
  ra_kde_desc d = legacy_desc(RA_LAYOUT_RAGGED, P, NX, NY, 0, 0, D, sigma, 1);
  const Layout L = make_layout(&d);
  int rc = check_common(&d, workspace, workspace_bytes, L.total);
  if (rc) return rc;
  ra_kde_inputs in;
  std::memset(&in, 0, sizeof(in));
  in.x = x;
  in.y = y;
  in.w_x = w_x;
  in.w_y = w_y;
  in.ptr_x = ptr_x;
  in.ptr_y = ptr_y;
  cudaStream_t st = (cudaStream_t)stream;
  double *Kt = at<double>(workspace, L.Ktmp);
  // the forward writes K into the workspace's Ktmp region
  rc = forward_impl(&d, &in, Kt, Kt + P, Kt + 2 * P, workspace, workspace_bytes, st);
  if (rc || P == 0) return rc;
  double *coef = at<double>(workspace, L.coef);
  mmd_coef_kernel<<<(unsigned)ceil_div(P, 256), 256, 0, st>>>(P, grad_loss, coef);
  ++g_launches;
  if (cudaGetLastError() != cudaSuccess) return RA_ERR_CUDA;
  ra_kde_grads g;
  g.grad_x = grad_x;
  g.grad_y = grad_y;
  g.grad_wx = grad_wx;
  g.grad_wy = grad_wy;
  g.grad_sigma = grad_sigma_pairs;
  return backward_impl(&d, &in, coef, &g, workspace, workspace_bytes, st);
}

int ra_kde_mmd_forward_segmented_noalloc(const float *x, const float *y, const float *w_x,
                                         const float *w_y, const int64_t *ptr_x,
                                         const int64_t *ptr_y, int64_t P, int64_t NX,
                                         int64_t NY, int32_t D, double sigma, double *Kxx,
                                         double *Kyy, double *Kxy, ra_stream_t stream) {
  const size_t need = ra_kde_mmd_forward_segmented_workspace_bytes(P, NX, NY, D);
  if (need == 0) return RA_ERR_INVALID_ARGUMENT;
  if (need > kNoallocScratchBytes) return RA_ERR_SCRATCH_LIMIT;
  void *scratch = nullptr;
  const int rc = noalloc_scratch_address(&scratch);
  if (rc) return rc;
  // the forward zeroes the scratch header itself; everything else it reads
  // is written earlier in the same call
  return ra_kde_mmd_forward_segmented(x, y, w_x, w_y, ptr_x, ptr_y, P, NX, NY, D, sigma, Kxx,
                                      Kyy, Kxy, scratch, kNoallocScratchBytes, stream);
}

int ra_kde_check_noalloc(ra_stream_t stream) {
  void *scratch = nullptr;
  const int rc = noalloc_scratch_address(&scratch);
  if (rc) return rc;
  return ra_kde_check(scratch, stream);
}

int ra_ptr_from_batch(const int64_t *batch, int64_t n, int64_t num_graphs, int64_t *ptr,
                      int *flags, ra_stream_t stream) {
  if (n < 0 || num_graphs < 0 || ptr == nullptr || flags == nullptr ||
      (n > 0 && batch == nullptr))
    return RA_ERR_INVALID_ARGUMENT;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(flags, 0, sizeof(int), st) != cudaSuccess) return RA_ERR_CUDA;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = ceil_div(n + 1, (int64_t)256), cap = (int64_t)(sms > 0 ? sms : 1) * 8;
  ptr_from_batch_kernel<<<(unsigned)(want < cap ? want : cap), 256, 0, st>>>(batch, n, num_graphs,
                                                                           ptr, flags);
  ++g_launches;
  return cuda_status(cudaGetLastError());
}

unsigned long long ra_kernel_launch_count(void) { return g_launches.load(); }

int ra_probe_fp32_peak(float *scratch, int64_t scratch_floats, int iters, double *ops_per_s,
                       ra_stream_t stream) {
  if (scratch == nullptr || ops_per_s == nullptr || iters <= 0) return RA_ERR_INVALID_ARGUMENT;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int threads = 256, blocks = sms * 8;
  if (scratch_floats < (int64_t)threads * blocks) return RA_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  cudaEvent_t e0, e1;
  if (cudaEventCreate(&e0) != cudaSuccess) return RA_ERR_CUDA;
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return RA_ERR_CUDA;
  }
  fp32_probe_kernel<<<blocks, threads, 0, st>>>(scratch, iters / 4 + 1, 1.0f);  // warm-up
  cudaEventRecord(e0, st);
  fp32_probe_kernel<<<blocks, threads, 0, st>>>(scratch, iters, 1.0f);
  cudaEventRecord(e1, st);
  g_launches += 2;
  int rc = RA_OK;
  if (cudaEventSynchronize(e1) != cudaSuccess) rc = RA_ERR_CUDA;
  float ms = 0.f;
  if (!rc && cudaEventElapsedTime(&ms, e0, e1) != cudaSuccess) rc = RA_ERR_CUDA;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (rc) return rc;
  // each fma2 = 2 FP32 lane operations
  const double ops = (double)blocks * threads * iters * 16.0 * 8.0 * 2.0;
  *ops_per_s = ops / (ms * 1e-3);
  return RA_OK;
}

// ---- float64 verification path (ra_exact.cuh) ------------------------------

size_t ra_kde_exact_workspace_bytes(int64_t NX, int64_t NY) {
  if (NX < 0 || NY < 0) return 0;
  return 256 + sizeof(double) * 4 * (size_t)(NX + NY);
}

int ra_kde_exact_f64(const double *x, const double *y, const double *w_x, const double *w_y,
                     const int64_t *ptr_x, const int64_t *ptr_y, int64_t P, int64_t NX,
                     int64_t NY, int32_t D, double sigma, double *loss, double *Kxx, double *Kyy,
                     double *Kxy, double *grad_x, double *grad_y, double *grad_wx,
                     double *grad_wy, double *grad_sigma, void *workspace,
                     size_t workspace_bytes, ra_stream_t stream) {
  if (P < 0 || NX < 0 || NY < 0 || D < 1 || D > kExactMaxD) return RA_ERR_INVALID_ARGUMENT;
  if (!(sigma > 0.0)) return RA_ERR_SIGMA;
  if (ptr_x == nullptr || ptr_y == nullptr || Kxx == nullptr || Kyy == nullptr ||
      Kxy == nullptr || workspace == nullptr)
    return RA_ERR_INVALID_ARGUMENT;
  if ((NX > 0 && (x == nullptr || w_x == nullptr)) || (NY > 0 && (y == nullptr || w_y == nullptr)))
    return RA_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < ra_kde_exact_workspace_bytes(NX, NY) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return RA_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  ExactArgs A;
  A.P = P;
  A.NX = NX;
  A.NY = NY;
  A.D = D;
  A.sigma = sigma;
  A.x = x;
  A.y = y;
  A.w_x = w_x;
  A.w_y = w_y;
  A.ptr_x = ptr_x;
  A.ptr_y = ptr_y;
  A.grad_x = grad_x;
  A.grad_y = grad_y;
  A.grad_wx = grad_wx;
  A.grad_wy = grad_wy;
  A.err = static_cast<int *>(workspace);
  A.work = reinterpret_cast<double *>(static_cast<char *>(workspace) + 256);
  // the ptr checks must pass before any kernel walks the segments: this
  // verification path synchronises the stream once to read them
  if (cudaMemsetAsync(A.err, 0, sizeof(int), st) != cudaSuccess) return RA_ERR_CUDA;
  exact_check_kernel<<<(unsigned)ceil_div(P + 1, (int64_t)256), 256, 0, st>>>(A);
  ++g_launches;
  int err = 0;
  if (cudaMemcpyAsync(&err, A.err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return RA_ERR_CUDA;
  if (err & kErrPtrStart) return RA_ERR_PTR_START;
  if (err & kErrPtrEnd) return RA_ERR_PTR_END;
  if (err & kErrPtrOrder) return RA_ERR_PTR_ORDER;
  if (P == 0) return RA_OK;
  if (NX + NY > 0) {
    exact_points_kernel<<<(unsigned)ceil_div(NX + NY, (int64_t)128), 128, 0, st>>>(A);
    ++g_launches;
  }
  exact_pairs_kernel<<<(unsigned)P, 256, 0, st>>>(A, Kxx, Kyy, Kxy, loss, grad_sigma);
  ++g_launches;
  return cuda_status(cudaGetLastError());
}

int ra_kde_exact_matrices_f64(const double *a, int64_t n, const double *b, int64_t m, int32_t D,
                              double sigma, double *G, double *diff, ra_stream_t stream) {
  if (n < 0 || m < 0 || D < 1 || D > kExactMaxD) return RA_ERR_INVALID_ARGUMENT;
  if (!(sigma > 0.0)) return RA_ERR_SIGMA;
  if ((n > 0 && a == nullptr) || (m > 0 && b == nullptr)) return RA_ERR_INVALID_ARGUMENT;
  if (n * m > ((int64_t)1 << 36)) return RA_ERR_INVALID_ARGUMENT;
  if (n == 0 || m == 0 || (G == nullptr && diff == nullptr)) return RA_OK;
  exact_matrices_kernel<<<(unsigned)ceil_div(n * m, (int64_t)256), 256, 0,
                          (cudaStream_t)stream>>>(a, n, b, m, D, sigma, G, diff);
  ++g_launches;
  return cuda_status(cudaGetLastError());
}

// ---- pairwise-distance spectrum loss (ra_pdl.cuh) ---------------------------

namespace {
struct PdlLayout {
  size_t temp, keys_in[2], keys_out[2], vals_in[2], vals_out[2], total;
};
bool pdl_layout(int64_t G, int64_t Ps, int64_t Pt, PdlLayout &L) {
  if (G < 0 || Ps < 0 || Pt < 0 || Ps > INT32_MAX || Pt > INT32_MAX || G > INT32_MAX)
    return false;
  size_t temp = 0;
  for (int64_t P : {Ps, Pt}) {
    size_t t = 0;
    if (P > 0 && cub::DeviceSegmentedSort::SortPairs(
                     nullptr, t, (const float *)nullptr, (float *)nullptr,
                     (const uint32_t *)nullptr, (uint32_t *)nullptr, (int)P, (int)G,
                     (const int64_t *)nullptr, (const int64_t *)nullptr) != cudaSuccess)
      return false;
    temp = t > temp ? t : temp;
  }
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = a256(o + bytes);
    return at;
  };
  L.temp = take(temp > 0 ? temp : 1);
  const int64_t P[2] = {Ps, Pt};
  for (int s = 0; s < 2; ++s) {
    L.keys_in[s] = take(sizeof(float) * (size_t)(P[s] > 0 ? P[s] : 1));
    L.keys_out[s] = take(sizeof(float) * (size_t)(P[s] > 0 ? P[s] : 1));
    L.vals_in[s] = take(sizeof(uint32_t) * (size_t)(P[s] > 0 ? P[s] : 1));
    L.vals_out[s] = take(sizeof(uint32_t) * (size_t)(P[s] > 0 ? P[s] : 1));
  }
  L.total = o;
  return true;
}
PdlSide pdl_side(const ra_pdl_cloud *c, void *ws, const PdlLayout &L, int s, bool sorted) {
  PdlSide S;
  S.pts = c->points;
  S.perm = c->perm;
  S.ptr = c->ptr;
  S.poff = c->pair_offsets;
  S.pairs = c->num_pairs;
  S.keys = at<float>(ws, sorted ? L.keys_out[s] : L.keys_in[s]);
  S.vals = at<uint32_t>(ws, sorted ? L.vals_out[s] : L.vals_in[s]);
  return S;
}
bool pdl_ok(const ra_pdl_cloud *c) {
  return c != nullptr && c->ptr != nullptr && c->pair_offsets != nullptr && c->num_pairs >= 0 &&
         (c->num_pairs == 0 || c->points != nullptr) && c->max_group <= 65536;
}
}  // namespace

size_t ra_pdl_workspace_bytes(int64_t G, int64_t pairs_src, int64_t pairs_tgt) {
  PdlLayout L;
  return pdl_layout(G, pairs_src, pairs_tgt, L) ? L.total : 0;
}

int ra_pdl_forward(const ra_pdl_cloud *src, const ra_pdl_cloud *tgt, int64_t G, int32_t D,
                   double *loss, void *workspace, size_t workspace_bytes, ra_stream_t stream) {
  if (G < 0 || D < 1 || !pdl_ok(src) || !pdl_ok(tgt) || (G > 0 && loss == nullptr))
    return RA_ERR_INVALID_ARGUMENT;
  PdlLayout L;
  if (!pdl_layout(G, src->num_pairs, tgt->num_pairs, L)) return RA_ERR_INVALID_ARGUMENT;
  if (workspace == nullptr || workspace_bytes < L.total ||
      (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return RA_ERR_WORKSPACE;
  if (G == 0) return RA_OK;
  cudaStream_t st = (cudaStream_t)stream;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const ra_pdl_cloud *cl[2] = {src, tgt};
  for (int s = 0; s < 2; ++s) {
    const int64_t P = cl[s]->num_pairs;
    if (P == 0) continue;
    PdlSide S = pdl_side(cl[s], workspace, L, s, false);
    const int64_t blocks = ceil_div(P, (int64_t)256);
    pdl_dist_kernel<<<(unsigned)(blocks < (int64_t)sms * 16 ? blocks : (int64_t)sms * 16), 256, 0,
                      st>>>(S, G, D);
    size_t temp = L.keys_in[0] - L.temp;  // capacity of the sort's temp region
    if (cub::DeviceSegmentedSort::SortPairs(
            at<void>(workspace, L.temp), temp, at<const float>(workspace, L.keys_in[s]),
            at<float>(workspace, L.keys_out[s]), at<const uint32_t>(workspace, L.vals_in[s]),
            at<uint32_t>(workspace, L.vals_out[s]), (int)P, (int)G, cl[s]->pair_offsets,
            cl[s]->pair_offsets + 1, st) != cudaSuccess)
      return RA_ERR_CUDA;
    g_launches += 2;
  }
  pdl_loss_kernel<<<(unsigned)G, 256, 0, st>>>(pdl_side(src, workspace, L, 0, true),
                                               pdl_side(tgt, workspace, L, 1, true), G, loss);
  ++g_launches;
  return cuda_status(cudaGetLastError());
}

int ra_pdl_backward(const ra_pdl_cloud *src, const ra_pdl_cloud *tgt, int64_t G, int32_t D,
                    const double *grad_loss, float *grad_src, float *grad_tgt, void *workspace,
                    size_t workspace_bytes, ra_stream_t stream) {
  if (G < 0 || D < 1 || !pdl_ok(src) || !pdl_ok(tgt) || (G > 0 && grad_loss == nullptr))
    return RA_ERR_INVALID_ARGUMENT;
  PdlLayout L;
  if (!pdl_layout(G, src->num_pairs, tgt->num_pairs, L)) return RA_ERR_INVALID_ARGUMENT;
  if (workspace == nullptr || workspace_bytes < L.total ||
      (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return RA_ERR_WORKSPACE;
  if (G == 0) return RA_OK;
  cudaStream_t st = (cudaStream_t)stream;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const PdlSide Sx = pdl_side(src, workspace, L, 0, true), Sy = pdl_side(tgt, workspace, L, 1, true);
  float *grads[2] = {grad_src, grad_tgt};
  const PdlSide *sides[2] = {&Sx, &Sy};
  for (int s = 0; s < 2; ++s) {
    if (grads[s] == nullptr || sides[s]->pairs == 0) continue;
    const int64_t blocks = ceil_div(sides[s]->pairs, (int64_t)256);
    pdl_grad_kernel<<<(unsigned)(blocks < (int64_t)sms * 16 ? blocks : (int64_t)sms * 16), 256, 0,
                      st>>>(*sides[s], *sides[1 - s], G, D, grad_loss, grads[s]);
    ++g_launches;
  }
  return cuda_status(cudaGetLastError());
}

}  // extern "C"
