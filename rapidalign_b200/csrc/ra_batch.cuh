// ra_batch.cuh -- ptr offsets of a sorted PyG-style batch vector, built on the
// device (rapidalign/kde.py:124-156: ptr[g] = first node of graph g,
// ptr[num_graphs] = number of nodes), with the checks the reference makes on
// the host turned into flag bits, so that no value has to be read back before
// the work that uses ptr is enqueued.
#pragma once

#include "ra_common.cuh"

namespace ra {

enum : int {
  kBatchUnsorted = 1,  // batch[i] < batch[i - 1] somewhere
  kBatchNegative = 2,  // batch[0] < 0
  kBatchCount = 4,     // batch[n - 1] + 1 != num_graphs (the caller's count is wrong)
};

// Node i in [0, n] writes ptr[g] = i for every g in (batch[i - 1], batch[i]]
// (batch[-1] = -1, batch[n] = num_graphs), clipped to [0, num_graphs].  For a
// sorted vector with ids in [0, num_graphs) every entry is written exactly
// once; otherwise the flags say so and ptr is not to be trusted.
__global__ void ptr_from_batch_kernel(const int64_t *__restrict__ batch, int64_t n, int64_t P,
                                      int64_t *__restrict__ ptr, int *flags) {
  int f = 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i <= n; i += stride) {
    const int64_t lo = i > 0 ? batch[i - 1] : -1;
    const int64_t hi = i < n ? batch[i] : P;
    if (i > 0 && i < n && hi < lo) f |= kBatchUnsorted;
    if (i == 0 && n > 0 && hi < 0) f |= kBatchNegative;
    if (i == n && n > 0 && lo + 1 != P) f |= kBatchCount;
    const int64_t g0 = lo + 1 > 0 ? lo + 1 : 0;
    const int64_t g1 = hi < P ? hi : P;
    for (int64_t g = g0; g <= g1; ++g) ptr[g] = i;
  }
  if (f) atomicOr(flags, f);
}

}  // namespace ra
