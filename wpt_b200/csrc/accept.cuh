// Speculative decoding's acceptance step on the GPU, WPT's rule
// (packages/wpt-inference/src/wpt_inference/__init__.py:173-179,210-222):
//   p_j = softmax(top_k_mask(scores_j / temperature))       (float32)
//   draft j is kept iff u_j * q_j[tok_j] < p_j[tok_j];
//   at the first rejection the row's last token is drawn from
//   normalize(max(0, p_j - q_j)); when every draft is kept, from p_n.
// The reference draws with torch.rand and torch.multinomial on the host,
// one scalar at a time; here the draws are inputs (uniforms (R, n) for the
// tests, resample (R,) for the last token) and the last token is the inverse
// CDF of the weights: the first index whose float64 running sum exceeds
// resample * total.
//
// accept_stats_kernel, one CTA per (row, position): x = scores / temperature;
// with top_k, the top_k-th largest x by a 4 x 8-bit radix select
// (ties kept, as `scores < v[..., [-1]]` keeps them); the maximum m and the
// sum Z of exp(x - m) over the kept x, in one pass over the row.
// accept_draw_kernel, one CTA per row: the decisions (one thread, a handful
// of lookups), then the draw: each thread sums its contiguous slice of the
// weights in float64, a block scan finds the slice where the running sum
// crosses resample * total, and that thread walks its slice.
#pragma once

#include "common.cuh"

namespace wpt {

constexpr int ACCEPT_THREADS = 1024;

struct AcceptParams {
  const float* scores;    // (R, n + 1, V)
  const int64_t* drafted; // (R, n)
  const float* q;         // (R, n, V) drafter probabilities
  const float* uniforms;  // (R, n)
  const float* resample;  // (R,)
  const int64_t* lengths; // (R,) drafts verified per row, or null (all n)
  float* stats;           // (R, n + 1, 3): m, Z, top-k threshold (scratch)
  int64_t* tokens;        // (R, n + 1), -1 padded
  int64_t* accepted;      // (R,)
  int R, n, V, top_k;
  float temperature;
};

__device__ __forceinline__ uint32_t accept_key(float x) {
  const uint32_t bits = __float_as_uint(x);
  return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}
__device__ __forceinline__ float accept_unkey(uint32_t key) {
  return __uint_as_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
}

// drafts verified in row i: lengths[i] clamped to 0 .. n, or n
__device__ __forceinline__ int accept_row_drafts(const AcceptParams& p, int i) {
  if (p.lengths == nullptr) return p.n;
  const int64_t len = p.lengths[i];
  return len < 0 ? 0 : (len > p.n ? p.n : static_cast<int>(len));
}

template <typename T>
__device__ __forceinline__ T block_sum(T v, T* s_red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  T total = 0;
  if (threadIdx.x < 32) {
    T w = threadIdx.x < blockDim.x / 32 ? s_red[threadIdx.x] : T(0);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
    if (threadIdx.x == 0) s_red[32] = w;
  }
  __syncthreads();
  total = s_red[32];
  __syncthreads();
  return total;
}

__device__ __forceinline__ float block_max(float v, float* s_red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float w = threadIdx.x < blockDim.x / 32 ? s_red[threadIdx.x] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (threadIdx.x == 0) s_red[32] = w;
  }
  __syncthreads();
  const float total = s_red[32];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(ACCEPT_THREADS) accept_stats_kernel(const AcceptParams p) {
  __shared__ uint32_t s_hist[256];
  __shared__ float s_red[33];
  __shared__ uint32_t s_sel[2];
  const int j = blockIdx.x, i = blockIdx.y;
  const int ni = accept_row_drafts(p, i);
  if (j > ni) return;
  const float* x = p.scores + (static_cast<int64_t>(i) * (p.n + 1) + j) * p.V;
  const float temp = p.temperature;
  // the top_k-th largest x (radix select over order keys), or -inf without top_k
  float thr = -INFINITY;
  if (p.top_k > 0 && p.top_k < p.V) {
    uint32_t prefix = 0, mask = 0;
    int remaining = p.top_k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += blockDim.x) s_hist[b] = 0;
      __syncthreads();
      for (int v = threadIdx.x; v < p.V; v += blockDim.x) {
        const uint32_t key = accept_key(x[v] / temp);
        if ((key & mask) == prefix) atomicAdd(&s_hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        uint32_t c[8];
        int sum = 0;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          c[b] = s_hist[255 - (lane * 8 + b)];
          sum += c[b];
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const int excl = incl - sum;
        if (excl < remaining && incl >= remaining) {
          int acc = excl;
#pragma unroll
          for (int b = 0; b < 8; ++b) {
            if (acc + static_cast<int>(c[b]) >= remaining) {
              s_sel[0] = 255 - (lane * 8 + b);
              s_sel[1] = static_cast<uint32_t>(acc);
              break;
            }
            acc += c[b];
          }
        }
      }
      __syncthreads();
      prefix |= s_sel[0] << shift;
      mask |= 255u << shift;
      remaining -= static_cast<int>(s_sel[1]);
      __syncthreads();
    }
    thr = accept_unkey(prefix);
  }
  // the maximum and the sum of exp(x - m) over the kept x in one pass: each
  // thread keeps a running (maximum, sum) and rescales its sum when its
  // maximum rises; the block combines them (16-byte loads when rows allow)
  float m = -INFINITY, z = 0.f;
  auto take = [&](float y) {
    if (!(y >= thr)) return;
    if (y > m) {
      z = z * expf(m - y) + 1.f;
      m = y;
    } else {
      z += expf(y - m);
    }
  };
  if ((p.V & 3) == 0) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int v = threadIdx.x; v < p.V / 4; v += blockDim.x) {
      const float4 f = __ldg(x4 + v);
      take(f.x / temp);
      take(f.y / temp);
      take(f.z / temp);
      take(f.w / temp);
    }
  } else {
    for (int v = threadIdx.x; v < p.V; v += blockDim.x) take(__ldg(x + v) / temp);
  }
  const float mb = block_max(m, s_red);
  z = block_sum(m == -INFINITY ? 0.f : z * expf(m - mb), s_red);
  m = mb;
  if (threadIdx.x == 0) {
    float* st = p.stats + (static_cast<int64_t>(i) * (p.n + 1) + j) * 3;
    st[0] = m;
    st[1] = z;
    st[2] = thr;
  }
}

// p_j[v] as the reference's float32 softmax gives it
__device__ __forceinline__ float accept_prob(const float* x, const float* st, int v, float temp) {
  const float y = x[v] / temp;
  return y >= st[2] ? expf(y - st[0]) / st[1] : 0.f;
}

__global__ void __launch_bounds__(ACCEPT_THREADS) accept_draw_kernel(const AcceptParams p) {
  __shared__ double s_scan[33];
  __shared__ int s_pick[2];
  const int i = blockIdx.x;
  const int ni = accept_row_drafts(p, i);
  const float temp = p.temperature;
  int64_t* tokens = p.tokens + static_cast<int64_t>(i) * (p.n + 1);
  if (threadIdx.x == 0) {
    int reject = -1;
    for (int j = 0; j < ni; ++j) {
      const int64_t tok = p.drafted[static_cast<int64_t>(i) * p.n + j];
      const float* x = p.scores + (static_cast<int64_t>(i) * (p.n + 1) + j) * p.V;
      const float* st = p.stats + (static_cast<int64_t>(i) * (p.n + 1) + j) * 3;
      const float pj = (tok >= 0 && tok < p.V) ? accept_prob(x, st, static_cast<int>(tok), temp) : 0.f;
      const float qj = (tok >= 0 && tok < p.V) ? p.q[(static_cast<int64_t>(i) * p.n + j) * p.V + tok] : 0.f;
      if (p.uniforms[static_cast<int64_t>(i) * p.n + j] * qj < pj) {
        tokens[j] = tok;
      } else {
        reject = j;
        break;
      }
    }
    s_pick[0] = reject;
  }
  __syncthreads();
  const int reject = s_pick[0];
  const int jd = reject >= 0 ? reject : ni;  // the position the last token is drawn at
  const float* x = p.scores + (static_cast<int64_t>(i) * (p.n + 1) + jd) * p.V;
  const float* st = p.stats + (static_cast<int64_t>(i) * (p.n + 1) + jd) * 3;
  const float* qv = reject >= 0 ? p.q + (static_cast<int64_t>(i) * p.n + jd) * p.V : nullptr;
  const int per = (p.V + ACCEPT_THREADS - 1) / ACCEPT_THREADS;
  const int v0 = threadIdx.x * per, v1 = min(p.V, v0 + per);
  double part = 0.0;
  for (int v = v0; v < v1; ++v) {
    float w = accept_prob(x, st, v, temp);
    if (qv) w = fmaxf(w - qv[v], 0.f);
    part += static_cast<double>(w);
  }
  // block exclusive scan of the slices' sums (float64)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double incl = part;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_scan[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    double w = lane < ACCEPT_THREADS / 32 ? s_scan[lane] : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < ACCEPT_THREADS / 32) s_scan[lane] = w;
  }
  if (threadIdx.x == 0) s_pick[1] = p.V - 1;
  __syncthreads();
  const double before = (warp > 0 ? s_scan[warp - 1] : 0.0) + incl - part;
  const double total = s_scan[ACCEPT_THREADS / 32 - 1];
  const double target = static_cast<double>(p.resample[i]) * total;
  if (before <= target && before + part > target) {  // the crossing is in this slice
    double cs = before;
    for (int v = v0; v < v1; ++v) {
      float w = accept_prob(x, st, v, temp);
      if (qv) w = fmaxf(w - qv[v], 0.f);
      cs += static_cast<double>(w);
      if (cs > target) {
        s_pick[1] = v;
        break;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int kept = reject >= 0 ? reject : ni;
    tokens[kept] = s_pick[1];
    for (int j = kept + 1; j <= p.n; ++j) tokens[j] = -1;
    p.accepted[i] = kept;
  }
}

}  // namespace wpt
