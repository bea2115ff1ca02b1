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
// accept_draw_kernel, one CTA per row: the decisions (one thread per draft,
// the first rejection by an atomic minimum), then the draw: float64 sums of
// 256-entry chunks of the weights (coalesced), a block scan finds the chunk
// where the running sum crosses resample * total, and one warp walks it.
#pragma once

#include <type_traits>

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
  // x / temperature is x itself at temperature 1: that case skips the division
  auto pass = [&](auto unit) {
    auto scaled = [&](float v) { return decltype(unit)::value ? v : v / temp; };
    if ((p.V & 3) == 0) {  // four 16-byte loads in flight per thread
      const float4* x4 = reinterpret_cast<const float4*>(x);
      const int n4 = p.V / 4;
      int v = threadIdx.x;
      for (; v + 3 * ACCEPT_THREADS < n4; v += 4 * ACCEPT_THREADS) {
        float4 f[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) f[u] = __ldg(x4 + v + u * ACCEPT_THREADS);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          take(scaled(f[u].x));
          take(scaled(f[u].y));
          take(scaled(f[u].z));
          take(scaled(f[u].w));
        }
      }
      for (; v < n4; v += ACCEPT_THREADS) {
        const float4 f = __ldg(x4 + v);
        take(scaled(f.x));
        take(scaled(f.y));
        take(scaled(f.z));
        take(scaled(f.w));
      }
    } else {
      for (int v = threadIdx.x; v < p.V; v += blockDim.x) take(scaled(__ldg(x + v)));
    }
  };
  if (temp == 1.f) {
    pass(std::true_type());
  } else {
    pass(std::false_type());
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
  const float y = temp == 1.f ? x[v] : x[v] / temp;
  return y >= st[2] ? expf(y - st[0]) / st[1] : 0.f;
}

// The draw's weight of vocabulary entry v: p_j[v], or max(0, p_j[v] - q_j[v])
// after a rejection (qv non-null). The row's statistics come in registers
// (m, 1 / Z, threshold); the weight scales by 1 / Z instead of dividing,
// which only moves the inverse CDF's boundaries by float32 rounding.
struct DrawRow {
  const float* x;
  const float* qv;
  float m, rz, thr, temp;
  __device__ __forceinline__ float weight(int v) const {
    const float y = temp == 1.f ? x[v] : x[v] / temp;
    float w = y >= thr ? expf(y - m) * rz : 0.f;
    if (qv) w = fmaxf(w - qv[v], 0.f);
    return w;
  }
};

// One CTA per row. The decisions: thread j < drafts tests draft j
// (u_j q_j[tok] < p_j[tok]) and a block vote finds the first rejection.
// The draw: the row's weights in chunks of DRAW_CHUNK consecutive entries
// (lane l of a warp takes entries 8l .. 8l + 7 of a chunk, so the warp's
// loads are coalesced), each chunk's float64 sum into shared memory; a
// block scan over the chunks finds the one where the running sum crosses
// resample * total, and one warp rescans that chunk to the entry.
constexpr int DRAW_CHUNK = 256;
__global__ void __launch_bounds__(ACCEPT_THREADS) accept_draw_kernel(const AcceptParams p) {
  extern __shared__ double s_chunk[];  // ceil(V / DRAW_CHUNK) chunk sums
  __shared__ double s_scan[33];
  __shared__ int s_pick[3];
  const int i = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  constexpr int WARPS = ACCEPT_THREADS / 32;
  const int ni = accept_row_drafts(p, i);
  const float temp = p.temperature;
  int64_t* tokens = p.tokens + static_cast<int64_t>(i) * (p.n + 1);
  if (t == 0) {
    s_pick[0] = ni;  // the first rejected draft, ni when every draft is kept
    s_pick[1] = p.V - 1;  // the drawn entry (the last when rounding leaves the target past the end)
    s_pick[2] = -1;  // the chunk the running sum crosses the target in
  }
  __syncthreads();
  for (int j = t; j < ni; j += ACCEPT_THREADS) {
    const int64_t tok = p.drafted[static_cast<int64_t>(i) * p.n + j];
    const float* xj = p.scores + (static_cast<int64_t>(i) * (p.n + 1) + j) * p.V;
    const float* stj = p.stats + (static_cast<int64_t>(i) * (p.n + 1) + j) * 3;
    const bool in = tok >= 0 && tok < p.V;
    const float pj = in ? accept_prob(xj, stj, static_cast<int>(tok), temp) : 0.f;
    const float qj = in ? p.q[(static_cast<int64_t>(i) * p.n + j) * p.V + tok] : 0.f;
    if (!(p.uniforms[static_cast<int64_t>(i) * p.n + j] * qj < pj)) atomicMin(&s_pick[0], j);
  }
  __syncthreads();
  const int kept = s_pick[0];
  const int reject = kept < ni ? kept : -1;
  for (int j = t; j < kept; j += ACCEPT_THREADS) tokens[j] = p.drafted[static_cast<int64_t>(i) * p.n + j];
  const float* st = p.stats + (static_cast<int64_t>(i) * (p.n + 1) + kept) * 3;
  DrawRow row;
  row.x = p.scores + (static_cast<int64_t>(i) * (p.n + 1) + kept) * p.V;
  row.qv = reject >= 0 ? p.q + (static_cast<int64_t>(i) * p.n + kept) * p.V : nullptr;
  row.m = st[0];
  row.rz = 1.f / st[1];
  row.thr = st[2];
  row.temp = temp;
  const int chunks = (p.V + DRAW_CHUNK - 1) / DRAW_CHUNK;
  // each warp sums its chunks, two at a time: lane l takes entries 8l .. 8l + 7
  for (int c = warp; c < chunks; c += 2 * WARPS) {
    double part[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int v0 = (c + u * WARPS) * DRAW_CHUNK + 8 * lane;
      float w[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) w[e] = v0 + e < p.V ? row.weight(v0 + e) : 0.f;
      part[u] = 0.0;
#pragma unroll
      for (int e = 0; e < 8; ++e) part[u] += static_cast<double>(w[e]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      part[0] += __shfl_xor_sync(0xffffffffu, part[0], o);
      part[1] += __shfl_xor_sync(0xffffffffu, part[1], o);
    }
    if (lane == 0) {
      s_chunk[c] = part[0];
      if (c + WARPS < chunks) s_chunk[c + WARPS] = part[1];
    }
  }
  __syncthreads();
  // block scan over the chunk sums: thread t takes chunks [t * per, (t + 1) * per)
  const int per = (chunks + ACCEPT_THREADS - 1) / ACCEPT_THREADS;
  const int c0 = t * per, c1 = min(chunks, c0 + per);
  double mine = 0.0;
  for (int c = c0; c < c1; ++c) mine += s_chunk[c];
  double incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_scan[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    double w = lane < WARPS ? s_scan[lane] : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < WARPS) s_scan[lane] = w;
  }
  __syncthreads();
  const double total = s_scan[WARPS - 1];
  const double target = static_cast<double>(p.resample[i]) * total;
  double before = (warp > 0 ? s_scan[warp - 1] : 0.0) + incl - mine;
  if (c0 < c1 && before <= target && before + mine > target) {  // the crossing is in one of these chunks
    for (int c = c0; c < c1; ++c) {
      if (before + s_chunk[c] > target) {
        s_pick[2] = c;
        s_scan[32] = before;
        break;
      }
      before += s_chunk[c];
    }
  }
  __syncthreads();
  // one warp walks the crossing chunk
  if (warp == 0 && (total > target)) {
    const int c = s_pick[2];
    if (c >= 0) {
      const int v0 = c * DRAW_CHUNK + 8 * lane;
      double w8[8];
      double part = 0.0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        w8[e] = v0 + e < p.V ? static_cast<double>(row.weight(v0 + e)) : 0.0;
        part += w8[e];
      }
      double lincl = part;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, lincl, o);
        if (lane >= o) lincl += y;
      }
      double cs = s_scan[32] + lincl - part;
      const unsigned hit = __ballot_sync(0xffffffffu, cs <= target && cs + part > target);
      if (hit != 0 && lane == __ffs(hit) - 1) {
        int pick = v0 + 7;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          cs += w8[e];
          if (cs > target) {
            pick = v0 + e;
            break;
          }
        }
        s_pick[1] = pick < p.V ? pick : p.V - 1;
      }
    }
  }
  __syncthreads();
  if (t == 0) {
    tokens[kept] = s_pick[1];
    for (int j = kept + 1; j <= p.n; ++j) tokens[j] = -1;
    p.accepted[i] = kept;
  }
}

}  // namespace wpt
