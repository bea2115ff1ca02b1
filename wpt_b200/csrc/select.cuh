// Top-k row selection of exact attention (HySparse2's oracle selection):
// for each query at position p, the top_k rows among rows 0 .. p - window
// by their largest log-weight over the heads,
//     score(n) = max_h (q_h . k_n * scale - lse_h),
// as pytorch_kernels.py:112-117 computes it (row count chosen_columns,
// :73-77; -1 where a query has fewer rows; rows in no particular order).
// The Triton form streams the candidates several times, recomputing q k^T
// in each counting pass (triton_kernels.py:393-508); here the scores are
// computed once on the tensor cores and kept in caller scratch, then one
// radix select per query reads them.
//
// score_kernel: S^T = K Q^T with the 128 keys of a tile as M and up to 256
// (query, head) columns as N (K tiles by TMA, Q once by TMA), S^T
// double-buffered in TMEM. Thread r of warps 0-3 owns key r: it reads its
// row of S^T 32 columns at a time and takes the running maximum over each
// query's H consecutive columns, writing one fp32 score per (query, key)
// (coalesced: consecutive threads, consecutive keys). Key tiles of a query
// group are split over gridDim.y; scores need no merge.
//
// topk_kernel: one CTA per query. Scores become order-preserving 32-bit
// keys; four 8-bit MSB-first histogram passes find the top_k-th key
// (the row is cached in shared memory when it fits); a block scan then
// writes every row above it and, among rows equal to it, the lowest row
// indices until top_k are chosen. Deterministic; ties resolve by row index.
#pragma once

#include <climits>

#include "common.cuh"

namespace wpt {

struct ScoreParams {
  const int64_t* positions;  // (B, T)
  const float* lse;          // (B, T, H): each head's log-sum-exp (natural log)
  float* scores;             // (B * T, ld) scratch
  int64_t ld;
  unsigned* status;
  int B, T, H, N, window, TQ, groups_per_row, chunk_tiles;
  float scale;
};

template <int NCOL, int STAGES>
struct ScoreLayout {
  static constexpr int C = 128, BN = 128;
  static constexpr int Q_BYTES = NCOL * C * 2;
  static constexpr int K_BYTES = BN * C * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = ((Q_BYTES + 1023) / 1024) * 1024;
  static constexpr int OFF_LSE = OFF_K + STAGES * K_BYTES;
  static constexpr int OFF_LAST = OFF_LSE + NCOL * 4;
  static constexpr int OFF_BAR = OFF_LAST + 256 * 4;
  static constexpr int NBAR = 1 + 2 * STAGES + 4;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16 + 1024;
  static constexpr int TMEM_COLS = 2 * NCOL <= 32 ? 32 : 2 * NCOL <= 64 ? 64 : 2 * NCOL <= 128 ? 128 : 2 * NCOL <= 256 ? 256 : 512;
};

template <int NCOL, int STAGES>
__global__ void __launch_bounds__(192, 1)
    score_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const ScoreParams p) {
  using L = ScoreLayout<NCOL, STAGES>;
  constexpr int C = L::C, BN = L::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sK = smem + L::OFF_K;
  float* s_lse = reinterpret_cast<float*>(smem + L::OFF_LSE);
  int* s_last = reinterpret_cast<int*>(smem + L::OFF_LAST);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + STAGES;
  uint64_t* s_full = k_empty + STAGES;
  uint64_t* s_free = s_full + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  int* s_maxlast = reinterpret_cast<int*>(smem + L::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = blockIdx.x, split = blockIdx.y;
  const int b = group / p.groups_per_row;
  const int t0 = (group - b * p.groups_per_row) * p.TQ;
  const int TQg = min(p.TQ, p.T - t0);

  if (threadIdx.x == 0) *s_maxlast = -1;
  __syncthreads();
  for (int tq = threadIdx.x; tq < TQg; tq += blockDim.x) {
    const int64_t pos = p.positions[static_cast<int64_t>(b) * p.T + t0 + tq];
    int64_t last = pos - p.window;
    if (last > p.N - 1) last = p.N - 1;
    if (last < -1) last = -1;
    s_last[tq] = static_cast<int>(last);
    atomicMax(s_maxlast, static_cast<int>(last));
  }
  for (int c = threadIdx.x; c < NCOL; c += blockDim.x) {
    const int tq = c / p.H, h = c - tq * p.H;
    // padding columns get +inf: their scores are -inf and never win a maximum
    s_lse[c] = tq < TQg ? p.lse[(static_cast<int64_t>(b) * p.T + t0 + tq) * p.H + h] : INFINITY;
  }
  __syncthreads();
  const int maxlast = *s_maxlast;
  const int tiles_total = maxlast >= 0 ? maxlast / BN + 1 : 0;
  const int tile0 = split * p.chunk_tiles;
  const int left = tiles_total - tile0;
  const int ntiles = left <= 0 ? 0 : (left < p.chunk_tiles ? left : p.chunk_tiles);
  if (ntiles == 0) return;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(k_empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(s_full + s, 1);
      mbar_init(s_free + s, 128);
    }
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(s_tmem, L::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 5 && lane == 0) {
    tma_prefetch(&tm_q);
    tma_prefetch(&tm_k);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 5) {
    if (lane == 0) {
      const int qrow0 = (b * p.T + t0) * p.H;
      mbar_expect_tx(q_full, L::Q_BYTES);
      tma_load_2d(sQ, &tm_q, q_full, 0, qrow0);
      tma_load_2d(sQ + NCOL * 128, &tm_q, q_full, 64, qrow0);
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % STAGES;
        if (j >= STAGES && !mbar_wait(k_empty + st, ((j / STAGES) & 1) ^ 1, p.status)) break;
        const int n0 = (tile0 + j) * BN;
        mbar_expect_tx(k_full + st, L::K_BYTES);
        tma_load_3d(sK + st * L::K_BYTES, &tm_k, k_full + st, 0, n0, b);
        tma_load_3d(sK + st * L::K_BYTES + BN * 128, &tm_k, k_full + st, 64, n0, b);
      }
    }
    __syncwarp();
  } else if (warp == 4) {
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16(128, NCOL, 0, 0);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK);
      bool ok = mbar_wait(q_full, 0, p.status);
      for (int j = 0; ok && j < ntiles; ++j) {
        const int st = j % STAGES;
        if (!(ok = mbar_wait(k_full + st, (j / STAGES) & 1, p.status))) break;
        if (j >= 2 && !(ok = mbar_wait(s_free + (j & 1), ((j >> 1) & 1) ^ 1, p.status))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C / 16; ++kk) {
          mma_ss(tmem + (j & 1) * NCOL,
                 sdesc_sw128(k_addr + st * L::K_BYTES + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 16, 1024),
                 sdesc_sw128(q_addr + (kk >> 2) * (NCOL * 128) + (kk & 3) * 32, 16, 1024), IDESC, kk > 0 ? 1u : 0u);
        }
        mma_commit(k_empty + st);
        mma_commit(s_full + (j & 1));
      }
    }
    __syncwarp();
  } else {
    const int r = threadIdx.x;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const int64_t rowbase = static_cast<int64_t>(b) * p.T + t0;
    for (int j = 0; j < ntiles; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(s_full + (j & 1), (j >> 1) & 1, p.status))) break;
      tc_fence_after();
      const int n = (tile0 + j) * BN + r;
      int tq = 0, next = p.H;
      float cur = -INFINITY;
#pragma unroll 1
      for (int c32 = 0; c32 < NCOL / 32 + (NCOL % 32 ? 1 : 0); ++c32) {
        float v[32];
        if constexpr (NCOL % 32 == 0) {
          uint32_t x[32];
          tmem_ld32(lane_addr + (j & 1) * NCOL + c32 * 32, x);
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = __uint_as_float(x[c]);
        } else {
          uint32_t x[16];
          tmem_ld16(lane_addr + (j & 1) * NCOL, x);
#pragma unroll
          for (int c = 0; c < 16; ++c) v[c] = __uint_as_float(x[c]);
#pragma unroll
          for (int c = 16; c < 32; ++c) v[c] = -INFINITY;
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int gc = c32 * 32 + c;
          if (gc < NCOL) {
            cur = fmaxf(cur, fmaf(v[c], p.scale, -s_lse[gc]));
            if (gc + 1 == next) {
              if (tq < TQg && n <= s_last[tq]) p.scores[(rowbase + tq) * p.ld + n] = cur;
              cur = -INFINITY;
              ++tq;
              next += p.H;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(s_free + (j & 1));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// ------------------------------------------------------------ radix select

__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t bits = __float_as_uint(x);
  return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}

constexpr int TOPK_THREADS = 512;

// Block-wide exclusive scan of one int per thread (TOPK_THREADS threads);
// returns this thread's prefix and sets *total.
__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < TOPK_THREADS / 32 ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < TOPK_THREADS / 32) s_warp[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const int before = (warp > 0 ? s_warp[warp - 1] : 0) + x - v;
  *total = s_warp[TOPK_THREADS / 32 - 1];
  __syncthreads();
  return before;
}

// One CTA per query: chosen[b, t, :K] from scores[b*T + t, 0 .. last].
__global__ void __launch_bounds__(TOPK_THREADS)
    topk_kernel(const float* __restrict__ scores, int64_t ld, const int64_t* __restrict__ positions,
                int64_t* __restrict__ chosen, int T, int N, int K, int window, int cache_cap) {
  extern __shared__ uint32_t s_keys[];  // cache_cap keys, then 256 histogram bins, then 32 scan slots
  uint32_t* s_hist = s_keys + cache_cap;
  int* s_warp = reinterpret_cast<int*>(s_hist + 256);
  __shared__ uint32_t s_sel[2];
  if (K <= 0) return;
  const int64_t row = blockIdx.x;
  const int64_t pos = positions[row];
  int64_t last = pos - window;
  if (last > N - 1) last = N - 1;
  const int count = last < 0 ? 0 : static_cast<int>(last + 1);
  int64_t* out = chosen + row * K;
  if (count <= K) {  // every candidate, in row order, then -1
    for (int i = threadIdx.x; i < K; i += blockDim.x) out[i] = i < count ? i : -1;
    return;
  }
  const float* src = scores + row * ld;
  const bool cached = count <= cache_cap;
  if (cached)
    for (int i = threadIdx.x; i < count; i += blockDim.x) s_keys[i] = order_key(src[i]);
  uint32_t prefix = 0, mask = 0;
  int remaining = K;  // how many of the top rows lie at or below the current prefix
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) s_hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < count; i += blockDim.x) {
      const uint32_t key = cached ? s_keys[i] : order_key(src[i]);
      if ((key & mask) == prefix) atomicAdd(&s_hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32) {  // the bin where the count from the top reaches `remaining`
      const int lane = threadIdx.x;
      uint32_t c[8];
      int sum = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c[i] = s_hist[255 - (lane * 8 + i)];
        sum += c[i];
      }
      int incl = sum;  // inclusive scan over lanes, high bins first
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const int excl = incl - sum;
      if (excl < remaining && incl >= remaining) {
        int acc = excl;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (acc + static_cast<int>(c[i]) >= remaining) {
            s_sel[0] = 255 - (lane * 8 + i);
            s_sel[1] = static_cast<uint32_t>(acc);
            break;
          }
          acc += c[i];
        }
      }
    }
    __syncthreads();
    prefix |= s_sel[0] << shift;
    mask |= 255u << shift;
    remaining -= static_cast<int>(s_sel[1]);
    __syncthreads();
  }
  // prefix is the K-th largest key; `remaining` rows equal to it are taken
  const uint32_t thr = prefix;
  const int above = K - remaining;
  const int per = (count + TOPK_THREADS - 1) / TOPK_THREADS;
  const int i0 = threadIdx.x * per, i1 = min(count, i0 + per);
  int gt = 0, eq = 0;
  for (int i = i0; i < i1; ++i) {
    const uint32_t key = cached ? s_keys[i] : order_key(src[i]);
    gt += key > thr;
    eq += key == thr;
  }
  int total;
  int gt_off = block_exclusive_scan(gt, s_warp, &total);
  int eq_off = block_exclusive_scan(eq, s_warp, &total);
  for (int i = i0; i < i1; ++i) {
    const uint32_t key = cached ? s_keys[i] : order_key(src[i]);
    if (key > thr) {
      out[gt_off++] = i;
    } else if (key == thr) {
      if (eq_off < remaining) out[above + eq_off] = i;
      ++eq_off;
    }
  }
}

}  // namespace wpt
