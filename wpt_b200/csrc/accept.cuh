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
// (row, position) finds it by a 4 x 8-bit radix select (ties kept, as
// `scores < v[..., [-1]]` keeps them) and writes the row's (m, Z) as its
// first segment. The draw: DRAW_CPS-chunk slices of each row, one CTA per
// slice. Every CTA of a row makes the row's decisions (one warp per draft,
// the first rejection by an atomic minimum; all CTAs get the same answer),
// sums its slice of the draw's weights in DRAW_CHUNK-entry float64 chunk
// sums, and the row's last CTA to finish (an arrival counter) scans the
// chunk sums to the crossing chunk and walks it to the entry with one warp.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace wpt {

constexpr int ACCEPT_THREADS = 1024;  // the top-k statistics kernel
constexpr int STAT_THREADS = 256;     // the segment statistics kernel
constexpr int STAT_SEG = 2048;        // entries of one statistics unit (one warp)
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
  float* thr;             // (R, n + 1) scratch: the top_k-th largest x (top-k mode)
  double* chunk_sum;      // (R, chunks) scratch: the draw's chunk sums
  unsigned* count;        // (R,) scratch: draw CTAs of the row that finished
  int64_t* tokens;        // (R, n + 1), -1 padded
  int64_t* accepted;      // (R,)
  int R, n, V, top_k;
  int S, chunks;          // segments and chunks per row
  float temperature;
};

// Byte offsets of the scratch regions inside the caller's buffer (each
// region 256-byte aligned); the last value is the buffer's size.
struct AcceptScratch {
  size_t part, thr, chunk_sum, count, bytes;
};
inline size_t accept_align(size_t x) { return (x + 255) / 256 * 256; }
inline AcceptScratch accept_scratch(int R, int n, int V) {
  const size_t positions = static_cast<size_t>(R) * (n + 1);
  const size_t S = (static_cast<size_t>(V) + STAT_SEG - 1) / STAT_SEG;
  const size_t chunks = (static_cast<size_t>(V) + DRAW_CHUNK - 1) / DRAW_CHUNK;
  AcceptScratch a;
  a.part = 0;
  a.thr = a.part + accept_align(positions * S * sizeof(float2));
  a.chunk_sum = a.thr + accept_align(positions * sizeof(float));
  a.count = a.chunk_sum + accept_align(static_cast<size_t>(R) * chunks * sizeof(double));
  a.bytes = a.count + accept_align(static_cast<size_t>(R) * sizeof(unsigned));
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

// Top-k mode: one CTA per (row, position) selects the threshold and reduces
// the kept x of the whole row; the row's (m, Z) becomes segment 0 and the
// other segments are empty.
__global__ void __launch_bounds__(ACCEPT_THREADS) accept_topk_stats_kernel(const AcceptParams p) {
  __shared__ uint32_t s_hist[256];
  __shared__ float s_red[33];
  __shared__ uint32_t s_sel[2];
  const int j = blockIdx.x, i = blockIdx.y;
  if (blockIdx.x == 0 && blockIdx.y == 0)
    for (int r = threadIdx.x; r < p.R; r += blockDim.x) p.count[r] = 0u;
  const int ni = accept_row_drafts(p, i);
  if (j > ni) return;
  const int64_t ij = static_cast<int64_t>(i) * (p.n + 1) + j;
  const float* x = p.scores + ij * p.V;
  const float temp = p.temperature;
  // the top_k-th largest x (radix select over order keys)
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
  const float thr = accept_unkey(prefix);
  // the maximum and the sum of exp(x - m) over the kept x: a running
  // (maximum, sum) per thread, rescaled when its maximum rises
  float m = -INFINITY, z = 0.f;
  for (int v = threadIdx.x; v < p.V; v += blockDim.x) {
    const float y = x[v] / temp;
    if (!(y >= thr)) continue;
    if (y > m) {
      z = z * expf(m - y) + 1.f;
      m = y;
    } else {
      z += expf(y - m);
    }
  }
  const float mb = block_max(m, s_red);
  z = block_sum(m == -INFINITY ? 0.f : z * expf(m - mb), s_red);
  for (int s = threadIdx.x; s < p.S; s += blockDim.x)
    p.part[ij * p.S + s] = s == 0 ? make_float2(mb, z) : make_float2(-INFINITY, 0.f);
  if (threadIdx.x == 0) p.thr[ij] = thr;
}

// Segment statistics: warp w of the grid reduces units w, w + warps, ...;
// unit u is segment u % S of position u / S. Lane l reads 16-byte vectors
// l, l + 32, ... of the segment, four in flight, in batches of 16 values.
template <bool GREEDY>
__global__ void __launch_bounds__(STAT_THREADS) accept_stats_kernel(const AcceptParams p) {
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * STAT_THREADS + threadIdx.x) >> 5;
  const int warps = (gridDim.x * STAT_THREADS) >> 5;
  if (blockIdx.x == 0)
    for (int r = threadIdx.x; r < p.R; r += blockDim.x) p.count[r] = 0u;
  const int64_t units = static_cast<int64_t>(p.R) * (p.n + 1) * p.S;
  const float temp = p.temperature;
  const bool unit_temp = temp == 1.f;
  const bool vec = (p.V & 3) == 0 && (reinterpret_cast<uintptr_t>(p.scores) & 15) == 0;
  for (int64_t u = warp; u < units; u += warps) {
    const int64_t ij = u / p.S;
    const int s = static_cast<int>(u - ij * p.S);
    const int i = static_cast<int>(ij / (p.n + 1)), j = static_cast<int>(ij - static_cast<int64_t>(i) * (p.n + 1));
    if (j > accept_row_drafts(p, i)) continue;  // a position past the row's drafts: never read
    const float* x = p.scores + ij * p.V;
    const int v0 = s * STAT_SEG, v1 = min(p.V, v0 + STAT_SEG);
    float m = -INFINITY, z = 0.f;
    if (vec) {
      const float4* x4 = reinterpret_cast<const float4*>(x);
      for (int b = v0 / 4 + lane; b < v1 / 4; b += 4 * 32) {
        float y[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int e = b + 32 * k;
          const float4 f = e < v1 / 4 ? __ldg(x4 + e) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
          y[4 * k] = f.x;
          y[4 * k + 1] = f.y;
          y[4 * k + 2] = f.z;
          y[4 * k + 3] = f.w;
        }
        // x / temperature; at temperature 1 the division is skipped (x itself)
        if (!unit_temp) {
#pragma unroll
          for (int k = 0; k < 16; ++k) y[k] = y[k] / temp;
        }
        accept_stat_batch<GREEDY>(m, z, y);
      }
    } else {
      for (int b = v0 + lane; b < v1; b += 4 * 32) {
        float y[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int e = b + 32 * k;
          y[k] = e < v1 ? (unit_temp ? __ldg(x + e) : __ldg(x + e) / temp) : -INFINITY;
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
    if (lane == 0) p.part[u] = a;
  }
}

// The statistics (m, Z) of position ij from its S segments, by one warp:
// the maximum, then the segments' sums rescaled to it (greedy: the counts
// of the segments whose maximum is it), summed in a fixed order and
// broadcast from lane 0, so every warp of every CTA gets the same bits for
// the same position.
__device__ __forceinline__ float2 accept_position_stats(const AcceptParams& p, int64_t ij, int lane) {
  const float2* part = p.part + ij * p.S;
  float m = -INFINITY;
  for (int s = lane; s < p.S; s += 32) m = fmaxf(m, part[s].x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float z = 0.f;
  if (accept_greedy(p)) {
    for (int s = lane; s < p.S; s += 32) {
      const float2 e = part[s];
      z += e.x == m ? e.y : 0.f;
    }
  } else if (m != -INFINITY) {
    for (int s = lane; s < p.S; s += 32) {
      const float2 e = part[s];
      z += e.y * expf(e.x - m);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
  return make_float2(m, __shfl_sync(0xffffffffu, z, 0));
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

// grid (R, slices). The decisions: warp w tests drafts w, w + DRAW_WARPS, ...
// (u_j q_j[tok] < p_j[tok]) and an atomic minimum finds the first
// rejection. The slice: chunks [y * DRAW_CPS, (y + 1) * DRAW_CPS) of the
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
  const bool radix = accept_radix(p), greedy = accept_greedy(p);
  if (t == 0) {
    s_pick[0] = ni;       // the first rejected draft, ni when every draft is kept
    s_pick[1] = p.V - 1;  // the drawn entry (the last when rounding leaves the target past the end)
    s_pick[2] = -1;       // the chunk the running sum crosses the target in
    s_pick[3] = 0;        // this CTA is the row's last to finish its slice
  }
  __syncthreads();
  for (int j = warp; j < ni; j += DRAW_WARPS) {
    const int64_t ij = static_cast<int64_t>(i) * (p.n + 1) + j;
    const float2 st = accept_position_stats(p, ij, lane);
    if (lane == 0) {
      const int64_t tok = p.drafted[static_cast<int64_t>(i) * p.n + j];
      float pj = 0.f, qj = 0.f;
      if (tok >= 0 && tok < p.V) {
        const float x = p.scores[ij * p.V + tok];
        const float y = temp == 1.f ? x : x / temp;
        const float thr = radix ? p.thr[ij] : (greedy ? st.x : -INFINITY);
        pj = y >= thr ? expf(y - st.x) / st.y : 0.f;
        qj = p.q[(static_cast<int64_t>(i) * p.n + j) * p.V + tok];
      }
      if (!(p.uniforms[static_cast<int64_t>(i) * p.n + j] * qj < pj)) atomicMin(&s_pick[0], j);
    }
  }
  __syncthreads();
  const int kept = s_pick[0];
  const int reject = kept < ni ? kept : -1;
  const int64_t ik = static_cast<int64_t>(i) * (p.n + 1) + kept;
  if (warp == 0) {
    const float2 st = accept_position_stats(p, ik, lane);
    if (lane == 0) {
      s_stat[0] = st.x;
      s_stat[1] = 1.f / st.y;
      s_stat[2] = radix ? p.thr[ik] : (greedy ? st.x : -INFINITY);
    }
  }
  __syncthreads();
  DrawRow row;
  row.x = p.scores + ik * p.V;
  row.qv = reject >= 0 ? p.q + (static_cast<int64_t>(i) * p.n + kept) * p.V : nullptr;
  row.m = s_stat[0];
  row.rz = s_stat[1];
  row.thr = s_stat[2];
  row.temp = temp;
  double* sums = p.chunk_sum + static_cast<int64_t>(i) * p.chunks;
  const int c_begin = blockIdx.y * DRAW_CPS, c_end = min(p.chunks, c_begin + DRAW_CPS);
  // each warp sums its chunks of the slice, two at a time
  for (int c = c_begin + warp; c < c_end; c += 2 * DRAW_WARPS) {
    double part[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int cu = c + u * DRAW_WARPS;
      const int v0 = cu * DRAW_CHUNK + 8 * lane;
      float w[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) w[e] = cu < c_end && v0 + e < p.V ? row.weight(v0 + e) : 0.f;
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
      sums[c] = part[0];
      if (c + DRAW_WARPS < c_end) sums[c + DRAW_WARPS] = part[1];
      __threadfence();
    }
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
