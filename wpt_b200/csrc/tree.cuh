// Ancestor masks of draft trees for tree-masked verification attention.
// One thread per (row, node): it walks from the node to its root through
// the parent array and sets bit j of the node's mask for every node j met
// (itself included). Parents must come before their children
// (parents[i] < i); a parent that does not ends the walk, so every walk
// takes at most n steps and never leaves the row's n entries. The same
// pass can write each node's position (its table row, base[b] + i), which
// verification attention reads.
#pragma once

#include <cstdint>

namespace wpt {

__global__ void tree_bits_kernel(const int64_t* __restrict__ parents, int64_t parents_stride, int64_t rows, int n,
                                 uint64_t* __restrict__ bits, const int64_t* __restrict__ base,
                                 int64_t* __restrict__ positions) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= rows * n) return;
  const int64_t row = t / n;
  const int i = static_cast<int>(t - row * n);
  const int64_t* par = parents + row * parents_stride;
  uint64_t mask = 0;
  int j = i;
  while (j >= 0) {
    mask |= uint64_t(1) << j;
    const int64_t up = par[j];
    if (up >= j) break;  // not before its child: the walk stops
    j = static_cast<int>(up);  // < j, and -1 (or any negative) ends the loop
  }
  bits[t] = mask;
  if (positions != nullptr) positions[t] = base[row] + i;  // node i sits at table row base + i
}

}  // namespace wpt
