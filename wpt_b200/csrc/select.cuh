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
// (query, head) columns as N (K tiles by TMA, Q by TMA per query group),
// S^T double-buffered in TMEM. Thread r of warps 0-3 owns key r: it reads its
// row of S^T 32 columns at a time and takes the running maximum over each
// query's H consecutive columns, writing one fp32 score per (query, key)
// (coalesced: consecutive threads, consecutive keys). Key tiles of a query
// group are split over gridDim.y; scores need no merge.
//
// topk_kernel: one CTA per query, or (fewer queries than SMs) a 2-CTA
// cluster per query, each CTA one half of the row. Scores become
// order-preserving 32-bit keys (cached in shared memory when the slice
// fits); a histogram over the keys' range (summed over the cluster) and a
// sort of the one bin that holds the top_k-th key find it (radix passes
// when that bin is crowded); a block scan then writes every row above it
// and, among rows equal to it, the lowest row indices until top_k are
// chosen. Deterministic; ties resolve by row index.
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
  int balanced;              // 1: the live key tiles of all groups split evenly over the grid
  float scale;
};

constexpr int SCORE_BAL_GROUPS = 1024;  // most query groups the balanced split takes

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
  static constexpr int OFF_PRE = OFF_MISC + 32;
  static constexpr int BYTES = OFF_PRE + (SCORE_BAL_GROUPS + 1) * 4 + 1024;
  static constexpr int TMEM_COLS = 2 * NCOL <= 32 ? 32 : 2 * NCOL <= 64 ? 64 : 2 * NCOL <= 128 ? 128 : 2 * NCOL <= 256 ? 256 : 512;
};

// Key tiles group g's queries read (rows 0 .. max over its queries of p - window).
__device__ __forceinline__ int score_group_tiles(const ScoreParams& p, int g, int* last_out) {
  const int b = g / p.groups_per_row;
  const int t0 = (g - b * p.groups_per_row) * p.TQ;
  const int TQg = min(p.TQ, p.T - t0);
  int maxlast = -1;
  for (int tq = 0; tq < TQg; ++tq) {
    int64_t last = p.positions[static_cast<int64_t>(b) * p.T + t0 + tq] - p.window;
    if (last > p.N - 1) last = p.N - 1;
    if (last < -1) last = -1;
    if (last_out) last_out[tq] = static_cast<int>(last);
    maxlast = max(maxlast, static_cast<int>(last));
  }
  return maxlast >= 0 ? maxlast / 128 + 1 : 0;
}

// A CTA's work is one or more segments: key tiles [tile0, tile0 + ntiles) of
// a query group. Grid (groups, splits): one segment, chunk_tiles of the
// group's tiles. Balanced (decode-sized calls): the groups' live tiles laid
// end to end and cut into gridDim.x equal ranges, so that rows of any
// lengths keep every CTA equally busy; a range spans one or more groups.
// Between segments the CTA drains (all roles meet at a barrier) and loads
// the next group's queries.
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
  int* s_seg = reinterpret_cast<int*>(smem + L::OFF_MISC + 4);  // group, tile0, ntiles of the segment
  int* s_pre = reinterpret_cast<int*>(smem + L::OFF_PRE);       // balanced: live tiles before group g

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = p.B * p.groups_per_row;
  griddep_wait();  // lse comes from the kernel before (programmatic dependent launch)

  // the CTA's range of work
  int64_t range_lo = 0, range_hi = 0;
  if (p.balanced) {
    // live tiles per group, then an in-place prefix sum: thread t sums a
    // contiguous run of groups, a warp scan and a pass over the six warps'
    // totals give each run's offset
    for (int g = threadIdx.x; g < groups; g += blockDim.x) s_pre[g + 1] = score_group_tiles(p, g, nullptr);
    __syncthreads();
    const int per = (groups + blockDim.x - 1) / blockDim.x;
    const int g0 = 1 + threadIdx.x * per, g1 = min(groups + 1, g0 + per);
    int run = 0;
    for (int g = g0; g < g1; ++g) run += s_pre[g];
    int incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) s_lse[warp] = __int_as_float(incl);  // the warps' totals, before s_lse is used
    __syncthreads();
    int offset = incl - run;
    for (int w = 0; w < warp; ++w) offset += __float_as_int(s_lse[w]);
    for (int g = g0; g < g1; ++g) {
      offset += s_pre[g];
      s_pre[g] = offset;
    }
    if (threadIdx.x == 0) s_pre[0] = 0;
    __syncthreads();
    const int64_t total = s_pre[groups];
    range_lo = total * blockIdx.x / gridDim.x;
    range_hi = total * (blockIdx.x + 1) / gridDim.x;
    if (range_lo >= range_hi) return;
  }

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

  bool ok = true;
  int jbase = 0;  // tiles of earlier segments: ring and TMEM phases run on across segments
  int g_next = 0;
  for (int seg = 0; ok; ++seg) {
    // the segment: thread 0 finds it, every thread reads it
    if (threadIdx.x == 0) {
      int g = -1, tile0 = 0, nt = 0;
      if (p.balanced) {
        // groups that end before the range, or have no live tile, hold no segment
        while (g_next < groups && (s_pre[g_next + 1] <= range_lo || s_pre[g_next + 1] == s_pre[g_next])) ++g_next;
        if (g_next < groups && s_pre[g_next] < range_hi) {
          g = g_next;
          const int64_t a = max(range_lo, static_cast<int64_t>(s_pre[g]));
          const int64_t e = min(range_hi, static_cast<int64_t>(s_pre[g + 1]));
          tile0 = static_cast<int>(a - s_pre[g]);
          nt = static_cast<int>(e - a);
          ++g_next;
        }
      } else if (seg == 0) {
        g = blockIdx.x;
        const int tiles_total = score_group_tiles(p, g, nullptr);
        tile0 = blockIdx.y * p.chunk_tiles;
        const int left = tiles_total - tile0;
        nt = left <= 0 ? 0 : min(left, p.chunk_tiles);
      }
      s_seg[0] = nt > 0 ? g : -1;
      s_seg[1] = tile0;
      s_seg[2] = nt;
    }
    __syncthreads();
    const int group = s_seg[0], tile0 = s_seg[1], ntiles = s_seg[2];
    if (group < 0) break;
    const int b = group / p.groups_per_row;
    const int t0 = (group - b * p.groups_per_row) * p.TQ;
    const int TQg = min(p.TQ, p.T - t0);
    if (threadIdx.x == 0) score_group_tiles(p, group, s_last);
    for (int c = threadIdx.x; c < NCOL; c += blockDim.x) {
      const int tq = c / p.H, h = c - tq * p.H;
      // padding columns get +inf: their scores are -inf and never win a maximum
      s_lse[c] = tq < TQg ? p.lse[(static_cast<int64_t>(b) * p.T + t0 + tq) * p.H + h] : INFINITY;
    }
    __syncthreads();

    if (warp == 5) {
      if (lane == 0) {
        const int qrow0 = (b * p.T + t0) * p.H;
        mbar_expect_tx(q_full, L::Q_BYTES);
        tma_load_2d(sQ, &tm_q, q_full, 0, qrow0);
        tma_load_2d(sQ + NCOL * 128, &tm_q, q_full, 64, qrow0);
        for (int jj = 0; jj < ntiles; ++jj) {
          const int j = jbase + jj, st = j % STAGES;
          if (j >= STAGES && !mbar_wait(k_empty + st, ((j / STAGES) & 1) ^ 1, p.status)) break;
          const int n0 = (tile0 + jj) * BN;
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
        bool mok = mbar_wait(q_full, seg & 1, p.status);
        for (int jj = 0; mok && jj < ntiles; ++jj) {
          const int j = jbase + jj, st = j % STAGES;
          if (!(mok = mbar_wait(k_full + st, (j / STAGES) & 1, p.status))) break;
          if (j >= 2 && !(mok = mbar_wait(s_free + (j & 1), ((j >> 1) & 1) ^ 1, p.status))) break;
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
      for (int jj = 0; jj < ntiles; ++jj) {
        const int j = jbase + jj;
        if (!__all_sync(0xffffffffu, mbar_wait(s_full + (j & 1), (j >> 1) & 1, p.status))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int n = (tile0 + jj) * BN + r;
        if (TQg == 1 && NCOL <= 64) {
          // one query (decode): the key's score is the maximum over all the
          // columns (padding columns give -inf), a tree over independent terms
          float w[NCOL];
          if constexpr (NCOL == 16) {
            uint32_t x[16];
            tmem_ld16(lane_addr + (j & 1) * NCOL, x);
#pragma unroll
            for (int c = 0; c < 16; ++c) w[c] = fmaf(__uint_as_float(x[c]), p.scale, -s_lse[c]);
          } else {
#pragma unroll
            for (int c32 = 0; c32 < NCOL / 32; ++c32) {
              uint32_t x[32];
              tmem_ld32(lane_addr + (j & 1) * NCOL + c32 * 32, x);
#pragma unroll
              for (int c = 0; c < 32; ++c) w[c32 * 32 + c] = fmaf(__uint_as_float(x[c]), p.scale, -s_lse[c32 * 32 + c]);
            }
          }
#pragma unroll
          for (int width = NCOL / 2; width > 0; width >>= 1) {
#pragma unroll
            for (int c = 0; c < width; ++c) w[c] = fmaxf(w[c], w[c + width]);
          }
          tc_fence_before();
          mbar_arrive(s_free + (j & 1));
          if (n <= s_last[0]) p.scores[rowbase * p.ld + n] = w[0];
          continue;
        }
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
    jbase += ntiles;
    // the segment is drained: its products were all read (or a wait failed)
    ok = __syncthreads_and(ok);
    tc_fence_after();
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

constexpr int TOPK_THREADS = 1024;

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

constexpr int SELECT_BINS = 2048;  // first-pass histogram bins
constexpr int SELECT_CAND = 4096;  // (key, row) pairs of the threshold's bin kept in shared memory

// Block-wide minimum and maximum of one key per thread.
__device__ __forceinline__ void block_minmax(uint32_t& lo, uint32_t& hi, uint32_t* s_red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if (lane == 0) {
    s_red[warp] = lo;
    s_red[32 + warp] = hi;
  }
  __syncthreads();
  lo = UINT_MAX;
  hi = 0;
  for (int w = 0; w < TOPK_THREADS / 32; ++w) {
    lo = min(lo, s_red[w]);
    hi = max(hi, s_red[32 + w]);
  }
  __syncthreads();
}

// SLICES CTAs per query (SLICES = 2: one thread-block cluster; CTA r takes
// the r-th contiguous slice of the row's candidates): chosen[b, t, :K] from
// scores[b*T + t, 0 .. last]. The K-th largest key: a histogram of the keys
// over SELECT_BINS equal ranges of [min key, max key] (a monotone map, so the
// bins are ordered; with two slices the minimum, maximum and histogram are
// summed over the cluster through distributed shared memory) finds the bin
// where the count from the top reaches K; the keys of that bin, usually a
// few dozen, are gathered (from both slices) and sorted in shared memory,
// the same on every CTA of the cluster. When that bin holds more than
// SELECT_CAND keys, four 8-bit radix passes over the whole row find the key
// instead. Each CTA then writes its slice's chosen rows at the offsets its
// partner's counts give.
template <int SLICES>
__global__ void __launch_bounds__(TOPK_THREADS)
    topk_kernel(const float* __restrict__ scores, int64_t ld, const int64_t* __restrict__ positions,
                int64_t* __restrict__ chosen, int T, int N, int K, int window, int cache_cap) {
  static_assert(SLICES == 1 || SLICES == 2, "one CTA or a pair per query");
  // dynamic shared memory: cache_cap keys, SELECT_BINS bins, SELECT_CAND
  // 8-byte candidates (8-byte aligned), 64 reduction slots
  extern __shared__ uint32_t s_keys[];
  uint32_t* s_hist = s_keys + cache_cap;
  uint64_t* s_cand = reinterpret_cast<uint64_t*>(s_hist + SELECT_BINS + (cache_cap & 1));
  int* s_warp = reinterpret_cast<int*>(s_cand + SELECT_CAND);
  __shared__ uint32_t s_sel[3];
  __shared__ int s_ncand;
  __shared__ uint32_t s_mm[2];  // this slice's minimum and maximum key
  __shared__ int s_tot[2];      // this slice's keys above the threshold and equal to it
  griddep_wait();  // the scores come from the kernel before (programmatic dependent launch)
  if (K <= 0) return;
  const int64_t row = blockIdx.x / SLICES;
  const uint32_t rank = SLICES > 1 ? cluster_rank() : 0u;
  const int64_t pos = positions[row];
  int64_t last = pos - window;
  if (last > N - 1) last = N - 1;
  const int count = last < 0 ? 0 : static_cast<int>(last + 1);
  int64_t* out = chosen + row * K;
  if (count <= K) {  // every candidate, in row order, then -1 (the same decision on both CTAs)
    if (rank == 0)
      for (int i = threadIdx.x; i < K; i += blockDim.x) out[i] = i < count ? i : -1;
    return;
  }
  // this CTA's slice of the candidates: rows [base, base + n_local)
  const int s_len = SLICES == 1 ? count : ((count + 1) / 2 + 3) & ~3;
  const int base = static_cast<int>(rank) * s_len;
  const int n_local = max(0, min(count, base + s_len) - base);
  const float* row_src = scores + row * ld;
  const float* src = row_src + base;
  const bool cached = n_local <= cache_cap;
  auto key_at = [&](int i) { return cached ? s_keys[i] : order_key(src[i]); };  // i: slice index
  uint32_t lo = UINT_MAX, hi = 0;
  // the slice's keys (16-byte loads, four in flight per thread) into shared
  // memory with their minimum and maximum
  const bool vec = cached && (ld & 3) == 0 && (reinterpret_cast<uintptr_t>(scores) & 15) == 0;
  const int n4 = vec ? n_local / 4 : 0;
  for (int i4 = threadIdx.x; i4 < n4; i4 += 4 * TOPK_THREADS) {
    float4 f[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      f[u] = i4 + u * TOPK_THREADS < n4 ? __ldg(reinterpret_cast<const float4*>(src) + i4 + u * TOPK_THREADS)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (i4 + u * TOPK_THREADS < n4) {
        const uint4 k4 = make_uint4(order_key(f[u].x), order_key(f[u].y), order_key(f[u].z), order_key(f[u].w));
        reinterpret_cast<uint4*>(s_keys)[i4 + u * TOPK_THREADS] = k4;
        lo = min(lo, min(min(k4.x, k4.y), min(k4.z, k4.w)));
        hi = max(hi, max(max(k4.x, k4.y), max(k4.z, k4.w)));
      }
    }
  }
  for (int i = 4 * n4 + threadIdx.x; i < n_local; i += blockDim.x) {
    const uint32_t key = order_key(src[i]);
    if (cached) s_keys[i] = key;
    lo = min(lo, key);
    hi = max(hi, key);
  }
  for (int i = threadIdx.x; i < SELECT_BINS; i += blockDim.x) s_hist[i] = 0;
  if (threadIdx.x == 0) s_ncand = 0;
  block_minmax(lo, hi, reinterpret_cast<uint32_t*>(s_warp));
  if constexpr (SLICES > 1) {  // the row's minimum and maximum over both slices
    if (threadIdx.x == 0) {
      s_mm[0] = lo;
      s_mm[1] = hi;
    }
    cluster_sync();
    const uint32_t other = dsmem_map(smem_u32(s_mm), rank ^ 1u);
    lo = min(lo, __float_as_uint(dsmem_ld(other)));
    hi = max(hi, __float_as_uint(dsmem_ld(other + 4)));
  }
  // bin(key) = floor((key - lo) * SELECT_BINS / (hi - lo + 1)) in float: monotone in key
  const float bscale = static_cast<float>(SELECT_BINS) / (static_cast<float>(hi - lo) + 1.f);
  auto bin_of = [&](uint32_t key) {
    return min(SELECT_BINS - 1, static_cast<int>(static_cast<float>(key - lo) * bscale));
  };
#pragma unroll 4
  for (int i = threadIdx.x; i < n_local; i += blockDim.x) atomicAdd(&s_hist[bin_of(key_at(i))], 1u);
  __syncthreads();
  // the bin where the count from the top reaches K: thread t sums bins
  // SELECT_BINS - 1 - (t * PER + e), e < PER, highest first (both slices')
  constexpr int PER = SELECT_BINS / TOPK_THREADS;
  if constexpr (SLICES > 1) cluster_sync();  // the partner's histogram is complete
  uint32_t hb[PER];
  int mine = 0;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const int bin = SELECT_BINS - 1 - (threadIdx.x * PER + e);
    hb[e] = s_hist[bin];
    if constexpr (SLICES > 1) hb[e] += __float_as_uint(dsmem_ld(dsmem_map(smem_u32(s_hist + bin), rank ^ 1u)));
    mine += static_cast<int>(hb[e]);
  }
  int total;
  const int before = block_exclusive_scan(mine, s_warp, &total);
  if (before < K && before + mine >= K) {
    int acc = before;
    for (int e = 0; e < PER; ++e) {
      const int bin = SELECT_BINS - 1 - (threadIdx.x * PER + e);
      if (acc + static_cast<int>(hb[e]) >= K) {
        s_sel[0] = static_cast<uint32_t>(bin);
        s_sel[1] = static_cast<uint32_t>(acc);  // keys in higher bins
        s_sel[2] = hb[e];                       // keys in this bin
        break;
      }
      acc += hb[e];
    }
  }
  __syncthreads();
  const int tbin = static_cast<int>(s_sel[0]);
  const int above_bin = static_cast<int>(s_sel[1]);
  const int nbin = static_cast<int>(s_sel[2]);
  // Slice rows are read in warp spans: warp w takes rows [w * span, (w + 1) *
  // span) of the slice, 32 at a time (lane l reads row base + l, so shared
  // memory serves a warp without bank conflicts); ballots rank keys inside a step.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int WARPS = TOPK_THREADS / 32;
  const int span = (n_local + WARPS - 1) / WARPS;
  const int w0 = min(n_local, warp * span), w1 = min(n_local, w0 + span);
  uint32_t thr;
  int remaining;       // keys equal to thr that are taken
  int gt = 0, eq = 0;  // this warp's keys above thr and equal to it
  if (nbin <= SELECT_CAND) {
    // one pass: the threshold bin's (key, row) pairs into shared memory, and
    // this warp's count of keys in higher bins
    if (threadIdx.x < 64) s_warp[threadIdx.x] = 0;
    int hi_w = 0;
#pragma unroll 4
    for (int b0 = w0; b0 < w1; b0 += 32) {
      const int i = b0 + lane;
      const uint32_t key = i < w1 ? key_at(i) : 0u;
      const int bin = i < w1 ? bin_of(key) : -1;
      hi_w += __popc(__ballot_sync(0xffffffffu, bin > tbin));
      if (bin == tbin)
        s_cand[atomicAdd(&s_ncand, 1)] = (static_cast<uint64_t>(key) << 32) | static_cast<uint32_t>(base + i);
    }
    __syncthreads();
    if constexpr (SLICES > 1) {
      // the partner's candidates after this slice's (together the bin's nbin
      // keys), then a barrier before either CTA sorts its copy in place
      cluster_sync();
      const int own = s_ncand;
      const uint32_t other_n = dsmem_map(smem_u32(&s_ncand), rank ^ 1u);
      const int theirs = static_cast<int>(__float_as_uint(dsmem_ld(other_n)));
      const uint32_t other_c = dsmem_map(smem_u32(s_cand), rank ^ 1u);
      for (int e = threadIdx.x; e < theirs; e += blockDim.x) {
        const uint32_t a = other_c + e * 8;
        s_cand[own + e] = static_cast<uint64_t>(__float_as_uint(dsmem_ld(a))) |
                          (static_cast<uint64_t>(__float_as_uint(dsmem_ld(a + 4))) << 32);
      }
      cluster_sync();
    }
    int size = 2;
    while (size < nbin) size <<= 1;
    for (int e = nbin + threadIdx.x; e < size; e += blockDim.x) s_cand[e] = 0ull;  // below every pair
    __syncthreads();
    // bitonic sort, descending
    for (int sp = 2; sp <= size; sp <<= 1) {
      for (int stride = sp >> 1; stride > 0; stride >>= 1) {
        for (int pr = threadIdx.x; pr < size / 2; pr += blockDim.x) {
          const int a = 2 * stride * (pr / stride) + (pr % stride), b2 = a + stride;
          const uint64_t ka = s_cand[a], kb = s_cand[b2];
          if ((a & sp) == 0 ? ka < kb : ka > kb) {
            s_cand[a] = kb;
            s_cand[b2] = ka;
          }
        }
        __syncthreads();
      }
    }
    const int need = K - above_bin;  // 1 .. nbin keys of the bin are taken
    thr = static_cast<uint32_t>(s_cand[need - 1] >> 32);
    int first = need - 1;  // the first position of thr in the sorted bin
    while (first > 0 && static_cast<uint32_t>(s_cand[first - 1] >> 32) == thr) --first;
    remaining = need - first;
    // this slice's keys of the bin above thr and equal to it, counted into their rows' warps
    for (int e = threadIdx.x; e < nbin; e += blockDim.x) {
      const uint32_t key = static_cast<uint32_t>(s_cand[e] >> 32);
      const int r = static_cast<int>(static_cast<uint32_t>(s_cand[e])) - base;
      if (r < 0 || r >= n_local) continue;
      const int w = r / span;
      if (key > thr) atomicAdd(&s_warp[w], 1);
      else if (key == thr) atomicAdd(&s_warp[32 + w], 1);
    }
    __syncthreads();
    gt = hi_w + s_warp[warp];
    eq = s_warp[32 + warp];
    __syncthreads();
  } else {  // a bin too full to gather: radix passes over all the row's keys
    if constexpr (SLICES > 1) cluster_sync();  // the partner has read this CTA's histogram
    auto row_key = [&](int i) {                // i: row index
      return SLICES == 1 ? key_at(i) : order_key(row_src[i]);
    };
    uint32_t prefix = 0, mask = 0;
    remaining = K;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = threadIdx.x; i < 256; i += blockDim.x) s_hist[i] = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < count; i += blockDim.x) {
        const uint32_t key = row_key(i);
        if ((key & mask) == prefix) atomicAdd(&s_hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (threadIdx.x < 32) {  // the bin where the count from the top reaches `remaining`
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
    thr = prefix;
#pragma unroll 4
    for (int b0 = w0; b0 < w1; b0 += 32) {
      const int i = b0 + lane;
      const uint32_t key = i < w1 ? key_at(i) : 0u;
      gt += __popc(__ballot_sync(0xffffffffu, i < w1 && key > thr));
      eq += __popc(__ballot_sync(0xffffffffu, i < w1 && key == thr));
    }
  }
  // every key above thr, and the `remaining` lowest-indexed keys equal to
  // it, in row order: the warps' counts (and, for the second slice, the
  // first slice's totals) place the warps
  const int above = K - remaining;
  if (lane == 0) {
    s_warp[warp] = gt;
    s_warp[32 + warp] = eq;
  }
  __syncthreads();
  int gt_off = 0, eq_off = 0;
  for (int v = 0; v < warp; ++v) {
    gt_off += s_warp[v];
    eq_off += s_warp[32 + v];
  }
  if constexpr (SLICES > 1) {
    if (threadIdx.x == 0) {
      int tg = 0, te = 0;
      for (int v = 0; v < WARPS; ++v) {
        tg += s_warp[v];
        te += s_warp[32 + v];
      }
      s_tot[0] = tg;
      s_tot[1] = te;
    }
    cluster_sync();
    if (rank == 1) {
      const uint32_t other = dsmem_map(smem_u32(s_tot), 0u);
      gt_off += static_cast<int>(__float_as_uint(dsmem_ld(other)));
      eq_off += static_cast<int>(__float_as_uint(dsmem_ld(other + 4)));
    }
  }
  const unsigned below = (1u << lane) - 1u;
#pragma unroll 4
  for (int b0 = w0; b0 < w1; b0 += 32) {
    const int i = b0 + lane;
    const uint32_t key = i < w1 ? key_at(i) : 0u;
    const bool is_gt = i < w1 && key > thr, is_eq = i < w1 && key == thr;
    const unsigned bg = __ballot_sync(0xffffffffu, is_gt), be = __ballot_sync(0xffffffffu, is_eq);
    if (is_gt) out[gt_off + __popc(bg & below)] = base + i;
    if (is_eq) {
      const int e = eq_off + __popc(be & below);
      if (e < remaining) out[above + e] = base + i;
    }
    gt_off += __popc(bg);
    eq_off += __popc(be);
  }
  if constexpr (SLICES > 1) cluster_sync();  // the partner has read this CTA's totals
}

}  // namespace wpt
