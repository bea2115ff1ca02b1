// Log-sum-exp merge of split-KV partial results.
//
// Each split s of a row (query, head) left o_s (its output normalised by its
// own softmax sum, fp32) and lse_s (natural log of that sum, -inf when the
// split saw no row). The whole row's result is
//     lse = log(sum_s exp(lse_s) + exp(sink_h))      (sink optional)
//     out = sum_s exp(lse_s - lse) o_s
// the same combination pytorch_kernels.py:183-184 makes over one block
// (logaddexp with the sink, weights exp(z - lse)). Used by the split-KV
// paths of both attention kernels and by the multi-GPU long-sequence decode,
// whose splits live on different GPUs.
#pragma once

#include "common.cuh"

namespace wpt {

// One warp per row; lane j handles columns j, j + 32, ...
template <int C>
__global__ void __launch_bounds__(256) merge_kernel(const float* __restrict__ part_o,
                                                    const float* __restrict__ part_lse, int splits,
                                                    int64_t rows, int64_t split_stride, int H,
                                                    const float* __restrict__ sink, __nv_bfloat16* __restrict__ out,
                                                    float* __restrict__ lse_out) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int h = static_cast<int>(row % H);
  float m = -INFINITY;
  for (int s = 0; s < splits; ++s) m = fmaxf(m, part_lse[s * split_stride + row]);
  const float sk = sink != nullptr ? sink[h] : -INFINITY;
  m = fmaxf(m, sk);
  float acc[C / 32];
#pragma unroll
  for (int i = 0; i < C / 32; ++i) acc[i] = 0.f;
  float denom = 0.f;
  if (m != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      const float ls = part_lse[s * split_stride + row];
      if (ls == -INFINITY) continue;
      const float w = __expf(ls - m);
      denom += w;
      const float* o = part_o + (s * split_stride + row) * C;
#pragma unroll
      for (int i = 0; i < C / 32; ++i) acc[i] = fmaf(w, o[lane + 32 * i], acc[i]);
    }
    if (sink != nullptr) denom += __expf(sk - m);
  }
  const float inv = denom > 0.f ? 1.f / denom : 0.f;
#pragma unroll
  for (int i = 0; i < C / 32; ++i) out[row * C + lane + 32 * i] = __float2bfloat16_rn(acc[i] * inv);
  if (lane == 0) lse_out[row] = denom > 0.f ? m + __logf(denom) : -INFINITY;
}

// The same merge for few rows with many splits (a long row split over many
// CTAs or GPUs): one CTA of MERGE_WARPS warps per row, warp w taking splits
// w, w + MERGE_WARPS, ..., the warps' maxima, sums and columns combined in
// shared memory, so the split loop is MERGE_WARPS times shorter.
constexpr int MERGE_WARPS = 8;
template <int C>
__global__ void __launch_bounds__(MERGE_WARPS * 32) merge_wide_kernel(
    const float* __restrict__ part_o, const float* __restrict__ part_lse, int splits, int64_t split_stride, int H,
    const float* __restrict__ sink, __nv_bfloat16* __restrict__ out, float* __restrict__ lse_out) {
  __shared__ float s_m[MERGE_WARPS], s_d[MERGE_WARPS];
  __shared__ float s_acc[MERGE_WARPS][C];
  const int64_t row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = static_cast<int>(row % H);
  float m = -INFINITY;
  for (int s = warp; s < splits; s += MERGE_WARPS) m = fmaxf(m, part_lse[s * split_stride + row]);
  if (lane == 0) s_m[warp] = m;
  __syncthreads();
  const float sk = sink != nullptr ? sink[h] : -INFINITY;
  m = sk;
#pragma unroll
  for (int w = 0; w < MERGE_WARPS; ++w) m = fmaxf(m, s_m[w]);
  float acc[C / 32];
#pragma unroll
  for (int i = 0; i < C / 32; ++i) acc[i] = 0.f;
  float denom = 0.f;
  if (m != -INFINITY) {
    for (int s = warp; s < splits; s += MERGE_WARPS) {
      const float ls = part_lse[s * split_stride + row];
      if (ls == -INFINITY) continue;
      const float wgt = __expf(ls - m);
      denom += wgt;
      const float* o = part_o + (s * split_stride + row) * C;
#pragma unroll
      for (int i = 0; i < C / 32; ++i) acc[i] = fmaf(wgt, o[lane + 32 * i], acc[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < C / 32; ++i) s_acc[warp][lane + 32 * i] = acc[i];
  if (lane == 0) s_d[warp] = denom;
  __syncthreads();
  if (warp == 0) {
    float d = (m != -INFINITY && sink != nullptr) ? __expf(sk - m) : 0.f;
#pragma unroll
    for (int w = 0; w < MERGE_WARPS; ++w) d += s_d[w];
    const float inv = d > 0.f ? 1.f / d : 0.f;
#pragma unroll
    for (int i = 0; i < C / 32; ++i) {
      float a = 0.f;
#pragma unroll
      for (int w = 0; w < MERGE_WARPS; ++w) a += s_acc[w][lane + 32 * i];
      out[row * C + lane + 32 * i] = __float2bfloat16_rn(a * inv);
    }
    if (lane == 0) lse_out[row] = d > 0.f ? m + __logf(d) : -INFINITY;
  }
}

}  // namespace wpt
