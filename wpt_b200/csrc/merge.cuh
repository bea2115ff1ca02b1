// Log-sum-exp merge of split-KV partial results.
//
// Each split s of a row (query, head) left o_s (its output normalised by its
// own softmax sum, fp32) and lse_s (natural log of that sum, -inf when the
// split saw no row). The whole row's result is
//     lse = log(sum_s exp(lse_s) + exp(sink_h))      (sink optional)
//     out = sum_s exp(lse_s - lse) o_s
// the same combination pytorch_kernels.py:183-184 makes over one block
// (logaddexp with the sink, weights exp(z - lse)). With out_f32 given, the
// output stays fp32 and, with no sink, the result is itself a partial (the
// normalised output of the splits together, and its log-sum) that a later
// merge can combine with others. Used by the split-KV
// paths of both attention kernels and by the multi-GPU long-sequence decode,
// whose splits live on different GPUs.
#pragma once

#include "common.cuh"

namespace wpt {

// Where split s's partials sit. Splits come in groups of `per` (one group
// per GPU of a long row, gathered side by side): within a group, split
// stride `stride` rows; group g's output partials start at g * group_o
// floats and its log-sums at g * group_l floats. One group (per = splits)
// is the plain (splits, rows) layout.
struct SplitLayout {
  int per;
  int64_t stride, group_o, group_l;
  __device__ __forceinline__ int64_t o(int s, int C) const {
    const int g = s / per;
    return g * group_o + (s - g * per) * stride * C;
  }
  __device__ __forceinline__ int64_t l(int s) const {
    const int g = s / per;
    return g * group_l + (s - g * per) * stride;
  }
};

// One warp per row; lane j handles columns j, j + 32, ... Splits are taken
// MERGE_BATCH at a time with all their loads (log-sums and output rows)
// issued together, in one online pass, so a row costs about one memory round
// trip per batch instead of one per split.
constexpr int MERGE_BATCH = 8;
template <int C>
__global__ void __launch_bounds__(256) merge_kernel(const float* __restrict__ part_o,
                                                    const float* __restrict__ part_lse, int splits,
                                                    int64_t rows, SplitLayout lay, int H,
                                                    const float* __restrict__ sink, __nv_bfloat16* __restrict__ out,
                                                    float* __restrict__ lse_out, float* __restrict__ out_f32) {
  griddep_wait();  // the partials come from the kernel before (programmatic dependent launch)
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int h = static_cast<int>(row % H);
  // one pass: each batch's log-sums and output rows are loaded together, and
  // the running maximum m (with acc and denom scaled to it) only rises
  const float sk = sink != nullptr ? sink[h] : -INFINITY;
  float m = sk;  // the sink joins the maximum (it is one more term of the denominator)
  float acc[C / 32];
#pragma unroll
  for (int i = 0; i < C / 32; ++i) acc[i] = 0.f;
  float denom = 0.f;
  for (int s0 = 0; s0 < splits; s0 += MERGE_BATCH) {
    float l8[MERGE_BATCH], o8[MERGE_BATCH][C / 32];
#pragma unroll
    for (int k = 0; k < MERGE_BATCH; ++k) {
      const int s = s0 + k;
      if (s < splits) {  // predicated: the batch's loads issue together
        l8[k] = part_lse[lay.l(s) + row];
        const float* o = part_o + lay.o(s, C) + row * C;
#pragma unroll
        for (int i = 0; i < C / 32; ++i) o8[k][i] = o[lane + 32 * i];
      } else {
        l8[k] = -INFINITY;
#pragma unroll
        for (int i = 0; i < C / 32; ++i) o8[k][i] = 0.f;
      }
    }
    float mb = m;
#pragma unroll
    for (int k = 0; k < MERGE_BATCH; ++k) mb = fmaxf(mb, l8[k]);
    if (mb != m) {  // the maximum rises: what is summed so far is rescaled (m = -inf: nothing summed yet)
      const float r = m == -INFINITY ? 0.f : __expf(m - mb);
      denom *= r;
#pragma unroll
      for (int i = 0; i < C / 32; ++i) acc[i] *= r;
      m = mb;
    }
#pragma unroll
    for (int k = 0; k < MERGE_BATCH; ++k) {
      if (l8[k] == -INFINITY) continue;  // an empty split's output row is not defined
      const float w = __expf(l8[k] - m);
      denom += w;
#pragma unroll
      for (int i = 0; i < C / 32; ++i) acc[i] = fmaf(w, o8[k][i], acc[i]);
    }
  }
  if (sink != nullptr && m != -INFINITY) denom += __expf(sk - m);
  const float inv = denom > 0.f ? 1.f / denom : 0.f;
  if (out_f32 != nullptr) {  // a partial of its own (normalised output, fp32) for a later merge
#pragma unroll
    for (int i = 0; i < C / 32; ++i) out_f32[row * C + lane + 32 * i] = acc[i] * inv;
  } else {
#pragma unroll
    for (int i = 0; i < C / 32; ++i) out[row * C + lane + 32 * i] = __float2bfloat16_rn(acc[i] * inv);
  }
  if (lane == 0) lse_out[row] = denom > 0.f ? m + __logf(denom) : -INFINITY;
}

// The same merge for few rows with many splits (a long row split over many
// CTAs or GPUs): one CTA of MERGE_THREADS per row. Its threads first take
// the splits' log-sums in parallel (maximum, weights into shared memory,
// their sum), then MERGE_THREADS / C groups of C threads each add a share of
// the splits' output rows (coalesced, several loads in flight per thread),
// and the groups' sums are combined in shared memory.
constexpr int MERGE_THREADS = 512, MERGE_MAX_SPLITS = 2048;
template <int C>
__global__ void __launch_bounds__(MERGE_THREADS) merge_wide_kernel(
    const float* __restrict__ part_o, const float* __restrict__ part_lse, int splits, SplitLayout lay, int H,
    const float* __restrict__ sink, __nv_bfloat16* __restrict__ out, float* __restrict__ lse_out,
    float* __restrict__ out_f32) {
  griddep_wait();  // the partials come from the kernel before (programmatic dependent launch)
  constexpr int GROUPS = MERGE_THREADS / C;
  __shared__ float s_w[MERGE_MAX_SPLITS];
  __shared__ int64_t s_off[MERGE_MAX_SPLITS];  // each split's output offset (floats) for this row
  __shared__ float s_red[MERGE_THREADS / 32 + 1];
  __shared__ float s_acc[GROUPS][C];
  const int64_t row = blockIdx.x;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int h = static_cast<int>(row % H);
  // maximum of the log-sums (and the sink)
  float m = -INFINITY;
  for (int s = t; s < splits; s += MERGE_THREADS) m = fmaxf(m, part_lse[lay.l(s) + row]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) s_red[warp] = m;
  __syncthreads();
  const float sk = sink != nullptr ? sink[h] : -INFINITY;
  m = sk;
#pragma unroll
  for (int w = 0; w < MERGE_THREADS / 32; ++w) m = fmaxf(m, s_red[w]);
  __syncthreads();
  // weights exp(lse_s - m) and their sum
  float d = 0.f;
  for (int s = t; s < splits; s += MERGE_THREADS) {
    const float ls = part_lse[lay.l(s) + row];
    const float w = (m == -INFINITY || ls == -INFINITY) ? 0.f : __expf(ls - m);
    s_w[s] = w;
    s_off[s] = lay.o(s, C);
    d += w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
  if (lane == 0) s_red[warp] = d;
  __syncthreads();
  // group g adds splits g, g + GROUPS, ...: thread c of the group, column c
  const int g = t / C, c = t - g * C;
  float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
  const float* o = part_o + row * C + c;
  int s = g;
  for (; s + 3 * GROUPS < splits; s += 4 * GROUPS) {
    const float w0 = s_w[s], w1 = s_w[s + GROUPS], w2 = s_w[s + 2 * GROUPS], w3 = s_w[s + 3 * GROUPS];
    const float o0 = w0 != 0.f ? o[s_off[s]] : 0.f;
    const float o1 = w1 != 0.f ? o[s_off[s + GROUPS]] : 0.f;
    const float o2 = w2 != 0.f ? o[s_off[s + 2 * GROUPS]] : 0.f;
    const float o3 = w3 != 0.f ? o[s_off[s + 3 * GROUPS]] : 0.f;
    acc0 = fmaf(w0, o0, acc0);
    acc1 = fmaf(w1, o1, acc1);
    acc2 = fmaf(w2, o2, acc2);
    acc3 = fmaf(w3, o3, acc3);
  }
  for (; s < splits; s += GROUPS) {
    const float w = s_w[s];
    if (w != 0.f) acc0 = fmaf(w, o[s_off[s]], acc0);
  }
  s_acc[g][c] = (acc0 + acc1) + (acc2 + acc3);
  __syncthreads();
  if (t < C) {
    float denom = (m != -INFINITY && sink != nullptr) ? __expf(sk - m) : 0.f;
#pragma unroll
    for (int w = 0; w < MERGE_THREADS / 32; ++w) denom += s_red[w];
    float a = 0.f;
#pragma unroll
    for (int k = 0; k < GROUPS; ++k) a += s_acc[k][t];
    const float inv = denom > 0.f ? 1.f / denom : 0.f;
    if (out_f32 != nullptr) {
      out_f32[row * C + t] = a * inv;
    } else {
      out[row * C + t] = __float2bfloat16_rn(a * inv);
    }
    if (t == 0) lse_out[row] = denom > 0.f ? m + __logf(denom) : -INFINITY;
  }
}

}  // namespace wpt
