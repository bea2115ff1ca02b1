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
// Two launches. The statistics: each position's row of x = scores /
// temperature is cut into STAT_SEG-entry segments and one warp reduces a
// segment to (maximum m_s, sum of exp(x - m_s)); the warps of the whole grid
// take the (row, position, segment) units in turn, so the logits stream from
// HBM through every SM with no tail of whole rows. top_k 1 (greedy) keeps
// the maxima: the units reduce to (maximum, count of maxima). A larger
// top_k's threshold needs the position's whole row: one CTA per
// (row, position) finds it (ties kept, as `scores < v[..., [-1]]` keeps
// them), reduces the kept x to (m, Z) and makes the draft's accept test.
// Of the segment units, the last of a position to finish (an arrival
// counter) combines its segments into (m, Z) and makes the accept test.
// The draw: DRAW_CPS-chunk slices of each row, one CTA per slice. Every CTA
// of a row finds the first failed test, sums its slice of the draw's
// weights in DRAW_CHUNK-entry float64 chunk sums, and the row's last CTA to
// finish (an arrival counter) scans the chunk sums to the crossing chunk and
// walks it to the entry with one warp.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace wpt {

constexpr int ACCEPT_THREADS = 1024;  // the top-k statistics kernel
constexpr int STAT_THREADS = 256;     // the segment statistics kernel
constexpr int STAT_SEG = 8192;        // entries of one statistics unit (one warp)
constexpr int STAT_VEC = 8;           // 16-byte loads a lane has in each batch (two batches in flight)
constexpr int DRAW_THREADS = 256;
constexpr int DRAW_WARPS = DRAW_THREADS / 32;
constexpr int DRAW_CHUNK = 256;       // entries of one float64 chunk sum
constexpr int DRAW_CPS = 32;          // chunks of one draw CTA's slice

struct AcceptParams {
  const float* scores;    // (R, n + 1, V)
  const int64_t* drafted; // (R, n)
  const float* q;         // (R, n, V) drafter probabilities
  const float* uniforms;  // (R, n)
  const float* resample;  // (R,)
  const int64_t* lengths; // (R,) drafts verified per row, or null (all n)
  float2* part;           // (R, n + 1, S) scratch: each segment's (maximum, sum of exp(x - maximum))
  float2* pos_stat;       // (R, n + 1) scratch: each position's (m, Z)
  float* thr;             // (R, n + 1) scratch: each position's threshold (top-k and greedy modes)
  int* keep;              // (R, n + 1) scratch: draft j's accept test passed (j < drafts of the row)
  double* chunk_sum;      // (R, chunks) scratch: the draw's chunk sums
  unsigned* pos_count;    // (R, n + 1) scratch, zeroed before the launches: segments of the position done
  unsigned* count;        // (R,) scratch, zeroed before the launches: draw CTAs of the row done
  unsigned long long* ticket;  // scratch, zeroed before the launches: statistics units taken
  int64_t* tokens;        // (R, n + 1), -1 padded
  int64_t* accepted;      // (R,)
  int R, n, V, top_k;
  int S, chunks;          // segments and chunks per row
  float temperature;
};

// Byte offsets of the scratch regions inside the caller's buffer (each
// region 256-byte aligned); the last value is the buffer's size.
struct AcceptScratch {
  size_t part, pos_stat, thr, keep, chunk_sum, pos_count, count, ticket, bytes;
};
inline size_t accept_align(size_t x) { return (x + 255) / 256 * 256; }
inline AcceptScratch accept_scratch(int R, int n, int V) {
  const size_t positions = static_cast<size_t>(R) * (n + 1);
  const size_t S = (static_cast<size_t>(V) + STAT_SEG - 1) / STAT_SEG;
  const size_t chunks = (static_cast<size_t>(V) + DRAW_CHUNK - 1) / DRAW_CHUNK;
  AcceptScratch a;
  a.part = 0;
  a.pos_stat = a.part + accept_align(positions * S * sizeof(float2));
  a.thr = a.pos_stat + accept_align(positions * sizeof(float2));
  a.keep = a.thr + accept_align(positions * sizeof(float));
  a.chunk_sum = a.keep + accept_align(positions * sizeof(int));
  a.pos_count = a.chunk_sum + accept_align(static_cast<size_t>(R) * chunks * sizeof(double));
  a.count = a.pos_count + positions * sizeof(unsigned);  // the counters are one zeroed range
  a.ticket = (a.count + static_cast<size_t>(R) * sizeof(unsigned) + 7) / 8 * 8;
  a.bytes = accept_align(a.ticket + sizeof(unsigned long long));
  return a;
}

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

// top_k 1 (greedy: p_j is uniform over the maxima of x): the statistics
// are (maximum, count of entries equal to it) and the threshold is the
// maximum. Larger top_k below V: the radix select of the top-k kernel.
__device__ __forceinline__ bool accept_greedy(const AcceptParams& p) { return p.top_k == 1 && p.V > 1; }
__device__ __forceinline__ bool accept_radix(const AcceptParams& p) { return p.top_k > 1 && p.top_k < p.V; }

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

// (maximum, sum) of two sets of exponentials, each relative to its own maximum
__device__ __forceinline__ float2 accept_stat_merge(float2 a, float2 b) {
  const float m = fmaxf(a.x, b.x);
  if (m == -INFINITY) return make_float2(-INFINITY, 0.f);
  return make_float2(m, a.y * expf(a.x - m) + b.y * expf(b.x - m));
}

// (maximum, count of entries equal to it) of two sets
__device__ __forceinline__ float2 accept_count_merge(float2 a, float2 b) {
  const float m = fmaxf(a.x, b.x);
  return make_float2(m, (a.x == m ? a.y : 0.f) + (b.x == m ? b.y : 0.f));
}

// A batch of K values into a running (maximum, sum): the sum is rescaled
// once per batch, when the batch raises the maximum. GREEDY: (maximum,
// count of entries equal to it) instead.
template <bool GREEDY, int K>
__device__ __forceinline__ void accept_stat_batch(float& m, float& z, const float (&y)[K]) {
  float bm = y[0];
#pragma unroll
  for (int k = 1; k < K; ++k) bm = fmaxf(bm, y[k]);
  if (GREEDY) {
    if (bm > m) {
      m = bm;
      z = 0.f;
    }
    if (bm == m) {
#pragma unroll
      for (int k = 0; k < K; ++k) z += y[k] == m ? 1.f : 0.f;
    }
    return;
  }
  if (bm == -INFINITY) return;  // nothing but -inf (exp gives 0)
  if (bm > m) {
    z *= expf(m - bm);
    m = bm;
  }
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < K; ++k) acc += expf(y[k] - m);
  z += acc;
}

// The statistics (m, Z) of position ij from its S segments, by one warp:
// the maximum, then the segments' sums rescaled to it (greedy: the counts
// of the segments whose maximum is it), summed in a fixed order and
// broadcast from lane 0, so every warp of every CTA gets the same bits for
// the same position.
__device__ __forceinline__ float2 accept_position_stats(const AcceptParams& p, int64_t ij, int lane) {
  const float2* part = p.part + ij * p.S;
  float m = -INFINITY;
  for (int s = lane; s < p.S; s += 32) m = fmaxf(m, __ldcg(&part[s]).x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float z = 0.f;
  if (accept_greedy(p)) {
    for (int s = lane; s < p.S; s += 32) {
      const float2 e = __ldcg(&part[s]);
      z += e.x == m ? e.y : 0.f;
    }
  } else if (m != -INFINITY) {
    for (int s = lane; s < p.S; s += 32) {
      const float2 e = __ldcg(&part[s]);
      z += e.y * expf(e.x - m);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
  return make_float2(m, __shfl_sync(0xffffffffu, z, 0));
}

// x / temperature as the reference's float32 division gives it, from the
// reciprocal r = 1 / t (correctly rounded) and Markstein's correction of
// the product: q0 = x r, then q0 + (x - q0 t) r with the remainder exact by
// fma (P. Markstein, IBM J. Res. Dev. 34(1), 1990). The remainder is exact,
// and the quotient the IEEE one, while it stays clear of float32's
// subnormal range: for quotients of magnitude 2^-100 and up. Below that it
// is within one unit in the last place (and exp(y - m) cannot tell). A zero,
// infinite or NaN q0 (signed zeros, masked -inf logits) is the quotient.
struct TempScale {
  float t, r;
  bool unit;
  __device__ __forceinline__ float operator()(float x) const {
    if (unit) return x;
    const float q0 = x * r;
    const float y = fmaf(fmaf(-q0, t, x), r, q0);
    const float a = fabsf(q0);
    return a < INFINITY && a > 0.f ? y : q0;
  }
};
__device__ __forceinline__ TempScale temp_scale(float t) {
  TempScale s;
  s.t = t;
  s.r = 1.f / t;
  s.unit = t == 1.f;
  return s;
}

__global__ void temperature_scale_kernel(const float* x, int64_t n, float t, float* out) {
  const TempScale scale = temp_scale(t);
  for (int64_t k = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; k < n;
       k += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[k] = scale(x[k]);
}

// Draft j's accept test, u_j q_j[tok] < p_j[tok], from its position's
// statistics: p_j[tok] = exp(y - m) / Z when y = x[tok] / temperature
// passes the threshold, else 0. A token outside the vocabulary fails.
__device__ __forceinline__ int accept_test(const AcceptParams& p, int64_t ij, int i, int j, float m, float z,
                                           float thr) {
  const int64_t tok = p.drafted[static_cast<int64_t>(i) * p.n + j];
  float pj = 0.f, qj = 0.f;
  if (tok >= 0 && tok < p.V) {
    const float y = temp_scale(p.temperature)(p.scores[ij * p.V + tok]);
    pj = y >= thr ? expf(y - m) / z : 0.f;
    qj = p.q[(static_cast<int64_t>(i) * p.n + j) * p.V + tok];
  }
  return p.uniforms[static_cast<int64_t>(i) * p.n + j] * qj < pj ? 1 : 0;
}

// The k-th largest of n order keys get(0) .. get(n - 1) by four 8-bit radix
// passes (every thread of the block calls it).
template <typename Get>
__device__ uint32_t block_radix_kth(Get get, int n, int k, uint32_t* s_hist, uint32_t* s_sel) {
  uint32_t prefix = 0, mask = 0;
  int remaining = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = threadIdx.x; b < 256; b += blockDim.x) s_hist[b] = 0;
    __syncthreads();
    for (int v = threadIdx.x; v < n; v += blockDim.x) {
      const uint32_t key = get(v);
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
  return prefix;
}

// Top-k mode (1 < top_k < V): one CTA per (row, position). Pass 1 takes
// each thread's maximum of its strided share of x and the row's maximum m;
// the top_k-th largest thread maximum t0 is a lower bound of the threshold
// (the maxima are some of the x). Pass 2 (from L2) gathers every x >= t0
// into shared memory, usually about top_k of them; a bitonic sort of their
// keys gives the threshold (the top_k-th largest, ties kept as
// `scores < v[..., [-1]]` keeps them) and Z = sum of exp(x - m) over the
// kept x, summed in sorted order. When more than TOPK_CAND pass t0 (or
// top_k exceeds the thread count), the threshold comes from radix passes
// over the whole row and (m, Z) from one more pass. The CTA writes the
// position's (m, Z), threshold and accept test.
constexpr int TOPK_CAND = 2048;
__global__ void __launch_bounds__(ACCEPT_THREADS) accept_topk_stats_kernel(const AcceptParams p) {
  __shared__ uint32_t s_hist[256];
  __shared__ float s_red[33];
  __shared__ uint32_t s_sel[2];
  __shared__ uint32_t s_keys[TOPK_CAND];
  __shared__ int s_count;
  const int j = blockIdx.x, i = blockIdx.y, t = threadIdx.x;
  griddep_launch();
  const int ni = accept_row_drafts(p, i);
  if (j > ni) return;
  const int64_t ij = static_cast<int64_t>(i) * (p.n + 1) + j;
  const float* x = p.scores + ij * p.V;
  const float temp = p.temperature;
  const TempScale scale = temp_scale(temp);
  auto y_at = [&](int v) { return scale(x[v]); };
  const int k = p.top_k;
  if (t == 0) s_count = 0;
  // pass 1: thread maxima and the row maximum
  float tm = -INFINITY;
  for (int v = t; v < p.V; v += ACCEPT_THREADS) tm = fmaxf(tm, y_at(v));
  const float m = block_max(tm, s_red);
  bool fast = k <= ACCEPT_THREADS;
  int count = 0;
  if (fast) {
    s_keys[t] = accept_key(tm);
    __syncthreads();
    const float t0 = accept_unkey(block_radix_kth([&](int v) { return s_keys[v]; }, ACCEPT_THREADS, k, s_hist, s_sel));
    // pass 2: every x at or above the bound (compared as floats, as the mask compares)
    for (int v = t; v < p.V; v += ACCEPT_THREADS) {
      const float y = y_at(v);
      if (y >= t0) {
        const int at = atomicAdd(&s_count, 1);
        if (at < TOPK_CAND) s_keys[at] = accept_key(y);
      }
    }
    __syncthreads();
    count = s_count;
    fast = count <= TOPK_CAND;
  }
  float thr, z;
  if (fast) {
    int size = 2;
    while (size < count) size <<= 1;
    for (int e = count + t; e < size; e += ACCEPT_THREADS) s_keys[e] = 0u;  // below every key
    __syncthreads();
    // bitonic sort, descending
    for (int span = 2; span <= size; span <<= 1) {
      for (int stride = span >> 1; stride > 0; stride >>= 1) {
        for (int pr = t; pr < size / 2; pr += ACCEPT_THREADS) {
          const int a = 2 * stride * (pr / stride) + (pr % stride), b = a + stride;
          const uint32_t ka = s_keys[a], kb = s_keys[b];
          const bool desc = (a & span) == 0;
          if (desc ? ka < kb : ka > kb) {
            s_keys[a] = kb;
            s_keys[b] = ka;
          }
        }
        __syncthreads();
      }
    }
    thr = accept_unkey(s_keys[k - 1]);
    float part = 0.f;
    for (int e = t; e < count; e += ACCEPT_THREADS) {
      const float y = accept_unkey(s_keys[e]);
      if (y >= thr) part += expf(y - m);
    }
    z = block_sum(part, s_red);
  } else {
    thr = accept_unkey(block_radix_kth([&](int v) { return accept_key(y_at(v)); }, p.V, k, s_hist, s_sel));
    // the sum of exp(x - m) over the kept x: a running (maximum, sum) per
    // thread, rescaled when its maximum rises
    float tmax = -INFINITY, tz = 0.f;
    for (int v = t; v < p.V; v += ACCEPT_THREADS) {
      const float y = y_at(v);
      if (!(y >= thr)) continue;
      if (y > tmax) {
        tz = tz * expf(tmax - y) + 1.f;
        tmax = y;
      } else {
        tz += expf(y - tmax);
      }
    }
    z = block_sum(tmax == -INFINITY ? 0.f : tz * expf(tmax - m), s_red);
  }
  if (t == 0) {
    p.pos_stat[ij] = make_float2(m, z);
    p.thr[ij] = thr;
    if (j < ni) p.keep[ij] = accept_test(p, ij, i, j, m, z, thr);
  }
}

// Segment statistics: warp w of the grid reduces units w, w + warps, ...;
// unit u is segment u % S of position u / S. Lane l reads 16-byte vectors
// l, l + 32, ... of the segment, four in flight, in batches of 16 values.
template <bool GREEDY, bool UNIT_TEMP>
__global__ void __launch_bounds__(STAT_THREADS) accept_stats_kernel(const AcceptParams p) {
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * STAT_THREADS + threadIdx.x) >> 5;
  const int warps = (gridDim.x * STAT_THREADS) >> 5;
  const int64_t units = static_cast<int64_t>(p.R) * (p.n + 1) * p.S;
  griddep_launch();
  const TempScale scale = temp_scale(p.temperature);
  const bool vec = (p.V & 3) == 0 && (reinterpret_cast<uintptr_t>(p.scores) & 15) == 0;
  // units: warp w starts with unit w, then takes tickets (one atomic per
  // unit, taken a unit ahead) so that warps on faster SMs take more units
  int64_t u = warp;
  while (u < units) {
    unsigned long long ticket = 0;
    if (lane == 0) ticket = atomicAdd(p.ticket, 1ull);
    const int64_t ij = u / p.S;
    const int s = static_cast<int>(u - ij * p.S);
    const int i = static_cast<int>(ij / (p.n + 1)), j = static_cast<int>(ij - static_cast<int64_t>(i) * (p.n + 1));
    const int ni = accept_row_drafts(p, i);
    const int64_t next = warps + static_cast<int64_t>(__shfl_sync(0xffffffffu, ticket, 0));
    if (j > ni) {  // a position past the row's drafts: never read
      u = next;
      continue;
    }
    const float* x = p.scores + ij * p.V;
    const int v0 = s * STAT_SEG, v1 = min(p.V, v0 + STAT_SEG);
    float m = -INFINITY, z = 0.f;
    if (vec) {  // lane l: 16-byte vectors l, l + 32, ... of the unit, in batches of STAT_VEC,
                // the next batch's loads in flight while a batch is reduced
      const float4* x4 = reinterpret_cast<const float4*>(x);
      const int e1 = v1 / 4;
      auto fetch = [&](int b, float4 (&f)[STAT_VEC]) {
#pragma unroll
        for (int k = 0; k < STAT_VEC; ++k) {
          const int e = b + 32 * k;
          f[k] = e < e1 ? __ldg(x4 + e) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        }
      };
      float4 cur[STAT_VEC], nxt[STAT_VEC];
      int b = v0 / 4 + lane;
      fetch(b, cur);
      for (; b < e1; b += STAT_VEC * 32) {
        fetch(b + STAT_VEC * 32, nxt);
        float y[4 * STAT_VEC];
#pragma unroll
        for (int k = 0; k < STAT_VEC; ++k) {
          y[4 * k] = cur[k].x;
          y[4 * k + 1] = cur[k].y;
          y[4 * k + 2] = cur[k].z;
          y[4 * k + 3] = cur[k].w;
        }
        if (!UNIT_TEMP) {
#pragma unroll
          for (int k = 0; k < 4 * STAT_VEC; ++k) y[k] = scale(y[k]);
        }
        accept_stat_batch<GREEDY>(m, z, y);
#pragma unroll
        for (int k = 0; k < STAT_VEC; ++k) cur[k] = nxt[k];
      }
    } else {  // lane l: entries l, l + 32, ...
      for (int b = v0 + lane; b < v1; b += 4 * 32) {
        float y[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int e = b + 32 * k;
          y[k] = e < v1 ? scale(__ldg(x + e)) : -INFINITY;
        }
        accept_stat_batch<GREEDY>(m, z, y);
      }
    }
    // the warp's (maximum, sum), combined in a fixed butterfly order
    float2 a = make_float2(m, z);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float2 b = make_float2(__shfl_xor_sync(0xffffffffu, a.x, o), __shfl_xor_sync(0xffffffffu, a.y, o));
      a = GREEDY ? accept_count_merge(a, b) : accept_stat_merge(a, b);
    }
    // the position's last segment to finish combines them and makes the
    // draft's accept test
    unsigned done = 0;
    if (lane == 0) {
      p.part[u] = a;
      __threadfence();
      done = atomicAdd(p.pos_count + ij, 1u);
    }
    if (__shfl_sync(0xffffffffu, done, 0) == static_cast<unsigned>(p.S - 1)) {
      __threadfence();
      const float2 st = accept_position_stats(p, ij, lane);
      if (lane == 0) {
        const float thr = GREEDY ? st.x : -INFINITY;
        p.pos_stat[ij] = st;
        p.thr[ij] = thr;
        if (j < ni) p.keep[ij] = accept_test(p, ij, i, j, st.x, st.y, thr);
      }
    }
    u = next;
  }
}

// The draw's weight of vocabulary entry v: p_j[v], or max(0, p_j[v] - q_j[v])
// after a rejection (qv non-null). The row's statistics come in registers
// (m, 1 / Z, threshold); the weight scales by 1 / Z instead of dividing,
// which only moves the inverse CDF's boundaries by float32 rounding.
// load8 reads entries v0 .. v0 + 7 (v0 a multiple of 8; two 16-byte loads
// each of x and q when the rows are 16-byte aligned); entries past the
// vocabulary read as x = -inf, q = 0, which weigh 0.
struct DrawRow {
  const float* x;
  const float* qv;
  float m, rz, thr;
  TempScale scale;
  bool vec;
  __device__ __forceinline__ void load8(int v0, int V, float (&xv)[8], float (&qq)[8]) const {
    if (vec && v0 + 8 <= V) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(x + v0));
      const float4 b = __ldg(reinterpret_cast<const float4*>(x + v0) + 1);
      xv[0] = a.x, xv[1] = a.y, xv[2] = a.z, xv[3] = a.w, xv[4] = b.x, xv[5] = b.y, xv[6] = b.z, xv[7] = b.w;
      if (qv) {
        const float4 c = __ldg(reinterpret_cast<const float4*>(qv + v0));
        const float4 d = __ldg(reinterpret_cast<const float4*>(qv + v0) + 1);
        qq[0] = c.x, qq[1] = c.y, qq[2] = c.z, qq[3] = c.w, qq[4] = d.x, qq[5] = d.y, qq[6] = d.z, qq[7] = d.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        xv[e] = v0 + e < V ? __ldg(x + v0 + e) : -INFINITY;
        if (qv) qq[e] = v0 + e < V ? __ldg(qv + v0 + e) : 0.f;
      }
    }
  }
  __device__ __forceinline__ float weight(float xe, float qe) const {
    const float y = scale(xe);
    float w = y >= thr ? expf(y - m) * rz : 0.f;
    if (qv) w = fmaxf(w - qe, 0.f);
    return w;
  }
};

// grid (R, slices). The first failed accept test (a ballot over the tests
// the statistics kernels made) gives the draw's position. The slice: chunks [y * DRAW_CPS, (y + 1) * DRAW_CPS) of the
// draw's weights, lane l of a warp taking entries 8l .. 8l + 7 of a chunk
// (coalesced), each chunk's float64 sum to the row's chunk sums. The row's
// last CTA to arrive scans the chunk sums for the one where the running sum
// crosses resample * total, and one warp rescans that chunk to the entry.
__global__ void __launch_bounds__(DRAW_THREADS) accept_draw_kernel(const AcceptParams p) {
  __shared__ double s_scan[DRAW_WARPS + 1];
  __shared__ int s_pick[4];
  __shared__ float s_stat[3];
  const int i = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int ni = accept_row_drafts(p, i);
  const float temp = p.temperature;
  const int64_t row0 = static_cast<int64_t>(i) * (p.n + 1);
  if (t == 0) {
    s_pick[1] = p.V - 1;  // the drawn entry (the last when rounding leaves the target past the end)
    s_pick[2] = -1;       // the chunk the running sum crosses the target in
    s_pick[3] = 0;        // this CTA is the row's last to finish its slice
  }
  griddep_wait();  // the statistics kernel's results
  // the first draft whose accept test failed (ni when every draft passed)
  if (warp == 0) {
    int first = ni;
    for (int j0 = 0; j0 < ni; j0 += 32) {
      const int j = j0 + lane;
      const unsigned failed = __ballot_sync(0xffffffffu, j < ni && p.keep[row0 + j] == 0);
      if (failed != 0) {
        first = j0 + __ffs(failed) - 1;
        break;
      }
    }
    if (lane == 0) {
      const float2 st = p.pos_stat[row0 + first];
      s_pick[0] = first;
      s_stat[0] = st.x;
      s_stat[1] = 1.f / st.y;
      s_stat[2] = p.thr[row0 + first];
    }
  }
  __syncthreads();
  const int kept = s_pick[0];
  const int reject = kept < ni ? kept : -1;
  const int64_t ik = row0 + kept;
  DrawRow row;
  row.x = p.scores + ik * p.V;
  row.qv = reject >= 0 ? p.q + (static_cast<int64_t>(i) * p.n + kept) * p.V : nullptr;
  row.m = s_stat[0];
  row.rz = s_stat[1];
  row.thr = s_stat[2];
  row.scale = temp_scale(temp);
  row.vec = (p.V & 3) == 0 && (reinterpret_cast<uintptr_t>(p.scores) & 15) == 0 &&
            (reinterpret_cast<uintptr_t>(p.q) & 15) == 0;
  double* sums = p.chunk_sum + static_cast<int64_t>(i) * p.chunks;
  const int c_begin = blockIdx.y * DRAW_CPS, c_end = min(p.chunks, c_begin + DRAW_CPS);
  // warp w sums chunks w, w + DRAW_WARPS, ... of the slice: every load first
  constexpr int CPW = DRAW_CPS / DRAW_WARPS;
  float xv[CPW][8], qq[CPW][8];
#pragma unroll
  for (int u = 0; u < CPW; ++u) {
    const int c = c_begin + warp + u * DRAW_WARPS;
    if (c < c_end) {
      row.load8(c * DRAW_CHUNK + 8 * lane, p.V, xv[u], qq[u]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) xv[u][e] = -INFINITY, qq[u][e] = 0.f;
    }
  }
  double part[CPW];
#pragma unroll
  for (int u = 0; u < CPW; ++u) {
    part[u] = 0.0;
#pragma unroll
    for (int e = 0; e < 8; ++e) part[u] += static_cast<double>(row.weight(xv[u][e], qq[u][e]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int u = 0; u < CPW; ++u) part[u] += __shfl_xor_sync(0xffffffffu, part[u], o);
  }
  if (lane == 0) {
#pragma unroll
    for (int u = 0; u < CPW; ++u) {
      const int c = c_begin + warp + u * DRAW_WARPS;
      if (c < c_end) sums[c] = part[u];
    }
    __threadfence();
  }
  __syncthreads();
  if (t == 0) {
    __threadfence();
    s_pick[3] = atomicAdd(p.count + i, 1u) == gridDim.y - 1 ? 1 : 0;
  }
  __syncthreads();
  if (!s_pick[3]) return;
  __threadfence();
  // the row's last CTA: block scan over the chunk sums, thread t taking
  // chunks [t * per, (t + 1) * per) (read from L2: other SMs wrote them)
  const int per = (p.chunks + DRAW_THREADS - 1) / DRAW_THREADS;
  const int c0 = t * per, c1 = min(p.chunks, c0 + per);
  double mine = 0.0;
  for (int c = c0; c < c1; ++c) mine += __ldcg(sums + c);
  double incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_scan[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    double w = lane < DRAW_WARPS ? s_scan[lane] : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < DRAW_WARPS) s_scan[lane] = w;
  }
  __syncthreads();
  const double total = s_scan[DRAW_WARPS - 1];
  const double target = static_cast<double>(p.resample[i]) * total;
  double before = (warp > 0 ? s_scan[warp - 1] : 0.0) + incl - mine;
  if (c0 < c1 && before <= target && before + mine > target) {  // the crossing is in one of these chunks
    for (int c = c0; c < c1; ++c) {
      const double sc = __ldcg(sums + c);
      if (before + sc > target) {
        s_pick[2] = c;
        s_scan[DRAW_WARPS] = before;
        break;
      }
      before += sc;
    }
  }
  __syncthreads();
  // one warp walks the crossing chunk
  if (warp == 0 && total > target) {
    const int c = s_pick[2];
    if (c >= 0) {
      const int v0 = c * DRAW_CHUNK + 8 * lane;
      float cx[8], cq[8];
      row.load8(v0, p.V, cx, cq);
      double w8[8];
      double part = 0.0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        w8[e] = static_cast<double>(row.weight(cx[e], cq[e]));
        part += w8[e];
      }
      double lincl = part;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, lincl, o);
        if (lane >= o) lincl += y;
      }
      double cs = s_scan[DRAW_WARPS] + lincl - part;
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
  int64_t* tokens = p.tokens + static_cast<int64_t>(i) * (p.n + 1);
  for (int j = t; j <= p.n; j += DRAW_THREADS)
    tokens[j] = j < kept ? p.drafted[static_cast<int64_t>(i) * p.n + j] : (j == kept ? s_pick[1] : -1);
  if (t == 0) p.accepted[i] = kept;
}

}  // namespace wpt
