// The generation cache's entries write: each row's new entries
// go after its earlier ones in the held table, the write of
// packages/wpt-model/src/wpt_model/cache.py:110-128 (Reading.everything)
// without its host synchronisations (the table's size and the list of
// written rows come from the host there: int(max) and nonzero). One warp
// per (row, new token): 16-byte copies of the entry. A row's new tokens past
// its count are padding and are not written; a destination past the table's
// capacity is not written either and sets the status word's shape bit.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace wpt {

__global__ void __launch_bounds__(256) cache_append_kernel(const uint8_t* __restrict__ src, int64_t src_sb,
                                                           int64_t src_sn, uint8_t* __restrict__ dst, int64_t dst_sb,
                                                           int64_t dst_sn, const int64_t* __restrict__ first,
                                                           const int64_t* __restrict__ counts, int B, int n,
                                                           int row_bytes, int64_t capacity, unsigned* status) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<int64_t>(B) * n) return;
  const int b = static_cast<int>(w / n), j = static_cast<int>(w - static_cast<int64_t>(b) * n);
  if (j >= counts[b]) return;  // padding
  const int64_t row = first[b] + j;
  if (row < 0 || row >= capacity) {
    if (lane == 0) atomicOr(status, STATUS_BAD_SHAPE);
    return;
  }
  const uint4* s = reinterpret_cast<const uint4*>(src + b * src_sb + static_cast<int64_t>(j) * src_sn);
  uint4* d = reinterpret_cast<uint4*>(dst + b * dst_sb + row * dst_sn);
  for (int i = lane; i < row_bytes / 16; i += 32) d[i] = s[i];
}

}  // namespace wpt
