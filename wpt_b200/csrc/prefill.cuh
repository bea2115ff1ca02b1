// Prefill / verification attention forward for one key-value head (MQA),
// tcgen05 + TMEM + TMA on sm_100a.
//
// Computes WPT's exact_attention output and log-sum-exp
// (packages/wpt-model/src/wpt_model/pytorch_kernels.py:98-121) for many
// queries per row, the window/sink form (pytorch_kernels.py:171-187 over a
// contiguous window; attention.py:85-107) and tree-masked verification.
//
// Tiles. A CTA owns BM = 128 "rows": TQ = 128 / H consecutive query tokens of
// one batch row, each with its H heads (row r = token r / H, head r % H).
// All heads of MQA read the same keys, so one K/V tile serves every row, and
// the 128 rows are the M of both products:
//   S  = Q K^T   M=128 rows, N=128 keys, K=C    A=Q (smem), B=K (smem)
//   O += P V     M=128 rows, N=C,       K=128  A=P (TMEM),  B=V (smem, MN-major)
// S is double-buffered in TMEM (2 x 128 columns), O takes C more columns; P
// (bf16) overwrites the first 64 columns of its S buffer.
//
// Warps: 0-3 softmax (thread = TMEM lane = row), 4 tcgen05 issuer (one lane),
// 5 TMA loader (one lane). Q arrives once; K and V tiles stream through
// STAGES shared-memory stages with separate full barriers so S can start
// before V lands.
//
// Online softmax in base 2 with a lazy maximum: a row's running maximum is
// only raised (and O rescaled) when a tile's maximum exceeds it by more
// than 8, so P stays below 2^8 and O is rarely touched. The rescale waits
// for the previous P V product to finish (o_done) and is done by every lane
// of a warp when any lane needs it (tcgen05.ld/st are warp-collective).
//
// Masks. Query t at position p (its own table row) reads rows lo..hi:
//   hi = min(p, N - 1); lo = max(0, p - window + 1 when window > 0, floor[b,t]).
// Tree mode adds: rows tree_base[b] + i (0 <= i < 64) are visible only when
// bit i of tree_bits[b, t] is set (node t sees itself and its ancestors).
// Tiles wholly inside a row's range skip the per-element mask.
//
// Split-KV: blockIdx.z splits the CTA's key tiles; with splits > 1 each
// split writes its normalised partial output and LSE (no sink) for the
// merge kernel, which adds the sink.
#pragma once

#include <climits>

#include "common.cuh"

namespace wpt {

struct PrefillParams {
  const int64_t* positions;   // (B, T) each query's own row
  const int64_t* floor_rows;  // (B, T) or null: lowest row each query may read
  const uint64_t* tree_bits;  // (B, T) or null: tree mode
  const int64_t* tree_base;   // (B,) or null: first row of the tree
  const float* sink;          // (H,) or null
  __nv_bfloat16* out;         // (B, T, H, C)
  float* lse;                 // (B, T, H)
  float* part_o;              // (splits, B*T*H, C) when splits > 1
  float* part_lse;            // (splits, B*T*H)
  unsigned* status;
  int B, T, H, N, window, TQ, splits;
  float scale_log2;  // softmax scale * log2(e)
};

template <int C, int STAGES>
struct PrefillLayout {
  static constexpr int BM = 128, BN = 128;
  static constexpr int SUB = C / 64;  // 64-element (128-byte) column chunks
  static constexpr int Q_BYTES = BM * C * 2;
  static constexpr int KV_BYTES = BN * C * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = Q_BYTES;
  static constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + STAGES * KV_BYTES;
  static constexpr int NBAR = 1 + 3 * STAGES + 6;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16 + 1024;  // + slack to align the base to 1024
};

__device__ __forceinline__ void prefill_query_rows(const PrefillParams& p, int b, int t, int& lo, int& hi) {
  const int64_t pos = p.positions[static_cast<int64_t>(b) * p.T + t];
  const int64_t top = pos < static_cast<int64_t>(p.N) - 1 ? pos : static_cast<int64_t>(p.N) - 1;
  int64_t low = 0;
  if (p.window > 0 && pos - p.window + 1 > low) low = pos - p.window + 1;
  if (p.floor_rows) {
    const int64_t f = p.floor_rows[static_cast<int64_t>(b) * p.T + t];
    if (f > low) low = f;
  }
  hi = top < -1 ? -1 : static_cast<int>(top);
  lo = low > INT_MAX ? INT_MAX : static_cast<int>(low);
}

template <int C, int STAGES>
__global__ void __launch_bounds__(192, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const PrefillParams p) {
  using L = PrefillLayout<C, STAGES>;
  constexpr int BM = L::BM, BN = L::BN, SUB = L::SUB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + STAGES;
  uint64_t* kv_empty = v_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;
  uint64_t* p_ready = s_full + 2;
  uint64_t* o_done = p_ready + 2;
  uint64_t* o_final = o_done + 1;  // one phase: the last P V product has completed
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  int* s_range = reinterpret_cast<int*>(smem + L::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qtile = gridDim.x - 1 - blockIdx.x;  // the last queries read the most rows: start them first
  const int b = blockIdx.y, split = blockIdx.z;
  const int t0 = qtile * p.TQ;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(kv_empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(s_full + s, 1);
      mbar_init(p_ready + s, 128);
    }
    mbar_init(o_done, 1);
    mbar_init(o_final, 1);
    fence_mbar_init();
    s_range[0] = INT_MAX;
    s_range[1] = -1;
  }
  if (warp == 4) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  if (warp == 5 && lane == 0) {
    tma_prefetch(&tm_q);
    tma_prefetch(&tm_k);
    tma_prefetch(&tm_v);
  }
  __syncthreads();
  if (static_cast<int>(threadIdx.x) < p.TQ && t0 + static_cast<int>(threadIdx.x) < p.T) {
    int lo, hi;
    prefill_query_rows(p, b, t0 + threadIdx.x, lo, hi);
    if (hi >= lo) {
      atomicMin(&s_range[0], lo);
      atomicMax(&s_range[1], hi);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  int tile0 = 0, ntiles = 0;
  {
    const int row_lo = s_range[0], row_hi = s_range[1];
    if (row_hi >= row_lo) {
      const int first = row_lo / BN, last = row_hi / BN, total = last - first + 1;
      const int per = (total + p.splits - 1) / p.splits;
      tile0 = first + split * per;
      const int left = last + 1 - tile0;
      ntiles = left < per ? (left > 0 ? left : 0) : per;
    }
  }

  if (warp == 5) {
    // ------------------------------------------------------------ TMA loader
    if (lane == 0 && ntiles > 0) {
      bool ok = true;
      int issued = 0;
      const int qrow0 = (b * p.T + t0) * p.H;
      mbar_expect_tx(q_full, L::Q_BYTES);
      for (int s = 0; s < SUB; ++s) tma_load_2d(sQ + s * BM * 128, &tm_q, q_full, s * 64, qrow0);
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % STAGES;
        const uint32_t use = j / STAGES;
        if (j >= STAGES && !(ok = mbar_wait(kv_empty + st, (use & 1) ^ 1, p.status))) break;
        const int n0 = (tile0 + j) * BN;
        mbar_expect_tx(k_full + st, L::KV_BYTES);
        for (int s = 0; s < SUB; ++s) tma_load_3d(sK + st * L::KV_BYTES + s * BN * 128, &tm_k, k_full + st, s * 64, n0, b);
        mbar_expect_tx(v_full + st, L::KV_BYTES);
        for (int s = 0; s < SUB; ++s) tma_load_3d(sV + st * L::KV_BYTES + s * BN * 128, &tm_v, v_full + st, s * 64, n0, b);
        issued = j + 1;
      }
      if (!ok) {  // let the copies in flight land before the CTA leaves
        mbar_wait(q_full, 0, p.status);
        for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j) {
          mbar_wait(k_full + j % STAGES, (j / STAGES) & 1, p.status);
          mbar_wait(v_full + j % STAGES, (j / STAGES) & 1, p.status);
        }
      }
    }
    __syncwarp();
  } else if (warp == 4) {
    // ------------------------------------------------------ tcgen05 issuer
    if (lane == 0 && ntiles > 0) {
      constexpr uint32_t IDESC_S = idesc_bf16(BM, BN, 0, 0);
      constexpr uint32_t IDESC_O = idesc_bf16(BM, C, 0, 1);
      const uint32_t tS = tmem, tO = tmem + 256;
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      bool ok = mbar_wait(q_full, 0, p.status);
      for (int j = 0; ok && j <= ntiles; ++j) {
        if (j < ntiles) {
          const int st = j % STAGES;
          if (!(ok = mbar_wait(k_full + st, (j / STAGES) & 1, p.status))) break;
          tc_fence_after();
          const uint32_t d = tS + (j & 1) * 128;
#pragma unroll
          for (int kk = 0; kk < C / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
            mma_ss(d, sdesc_sw128(q_addr + off, 16, 1024),
                   sdesc_sw128(k_addr + st * L::KV_BYTES + off, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
          }
          mma_commit(s_full + (j & 1));
        }
        if (j > 0) {
          const int jp = j - 1, st = jp % STAGES;
          if (!(ok = mbar_wait(p_ready + (jp & 1), (jp >> 1) & 1, p.status))) break;
          if (!(ok = mbar_wait(v_full + st, (jp / STAGES) & 1, p.status))) break;
          tc_fence_after();
          const uint32_t a = tS + (jp & 1) * 128;
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            mma_ts(tO, a + kk * 8, sdesc_sw128(v_addr + st * L::KV_BYTES + kk * 16 * 128, BN * 128, 1024), IDESC_O,
                   (jp > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(kv_empty + st);
          mma_commit(o_done);
          if (j == ntiles) mma_commit(o_final);
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------- softmax: one thread per row
    const int row = threadIdx.x;
    const int tq = row / p.H, h = row - tq * p.H;
    const int t = t0 + tq;
    const bool valid = tq < p.TQ && t < p.T;
    int lo = 0, hi = -1;
    if (valid) prefill_query_rows(p, b, t, lo, hi);
    int64_t tbase = int64_t(1) << 62;  // no tree: a base no row reaches
    uint64_t tbits = ~0ull;
    if (valid && p.tree_bits) {
      tbase = p.tree_base[b];
      tbits = p.tree_bits[static_cast<int64_t>(b) * p.T + t];
    }
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const uint32_t tO = lane_addr + 256;
    const float sl2 = p.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(s_full + (j & 1), (j >> 1) & 1, p.status));
      if (!ok) break;
      tc_fence_after();
      const int n0 = (tile0 + j) * BN;
      const uint32_t sAddr = lane_addr + (j & 1) * 128;
      float s[BN];
#pragma unroll
      for (int c4 = 0; c4 < BN / 32; ++c4) {
        uint32_t r[32];
        tmem_ld32(sAddr + c4 * 32, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c4 * 32 + i] = __uint_as_float(r[i]);
      }
      const bool whole = valid && n0 >= lo && n0 + BN - 1 <= hi &&
                         (static_cast<int64_t>(n0) + BN - 1 < tbase || static_cast<int64_t>(n0) >= tbase + 64);
      float tmax = -INFINITY;
      if (whole) {
#pragma unroll
        for (int i = 0; i < BN; ++i) tmax = fmaxf(tmax, s[i]);
      } else {
#pragma unroll
        for (int i = 0; i < BN; ++i) {
          const int n = n0 + i;
          bool vis = valid && n >= lo && n <= hi;
          const int64_t d = static_cast<int64_t>(n) - tbase;
          if (d >= 0 && d < 64) vis = vis && ((tbits >> d) & 1ull);
          s[i] = vis ? s[i] : -INFINITY;
          tmax = fmaxf(tmax, s[i]);
        }
      }
      tmax *= sl2;
      const bool need = tmax > m_used + 8.f;
      const float alpha = need ? fast_exp2(m_used - tmax) : 1.f;
      if (__any_sync(0xffffffffu, need) && j > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(o_done, (j - 1) & 1, p.status));
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int c4 = 0; c4 < C / 32; ++c4) {
          uint32_t r[32];
          tmem_ld32(tO + c4 * 32, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st32(tO + c4 * 32, r);
        }
      }
      if (need) {
        l *= alpha;
        m_used = tmax;
      }
      const float msub = m_used == -INFINITY ? 0.f : m_used;
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2) {
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float e0 = fast_exp2(fmaf(s[c2 * 64 + 2 * i], sl2, -msub));
          const float e1 = fast_exp2(fmaf(s[c2 * 64 + 2 * i + 1], sl2, -msub));
          l += e0 + e1;
          pk[i] = pack_bf16(e0, e1);
        }
        tmem_st32(sAddr + c2 * 32, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_ready + (j & 1));
    }
    // o_done's parity cannot name the last product here (the MMA may still be
    // two products behind, and phase ntiles - 3 has the same parity), so the
    // epilogue waits on o_final, which completes once, after the last one
    if (ok && ntiles > 0) ok = __all_sync(0xffffffffu, mbar_wait(o_final, 0, p.status));
    tc_fence_after();
    if (ok) {
      const int64_t orow = (static_cast<int64_t>(b) * p.T + t) * p.H + h;
      const float msub = m_used == -INFINITY ? 0.f : m_used;
      if (p.splits == 1) {
        float denom = l;
        if (p.sink != nullptr && valid) denom += fast_exp2(fmaf(p.sink[h], LOG2E, -msub));
        const float inv = denom > 0.f ? 1.f / denom : 0.f;
#pragma unroll
        for (int c4 = 0; c4 < C / 32; ++c4) {
          uint32_t r[32];
          if (ntiles > 0) {
            tmem_ld32(tO + c4 * 32, r);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = 0u;
          }
          if (valid) {
            uint4* dst = reinterpret_cast<uint4*>(p.out + orow * C + c4 * 32);
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
              uint4 w;
              w.x = pack_bf16(__uint_as_float(r[v4 * 8 + 0]) * inv, __uint_as_float(r[v4 * 8 + 1]) * inv);
              w.y = pack_bf16(__uint_as_float(r[v4 * 8 + 2]) * inv, __uint_as_float(r[v4 * 8 + 3]) * inv);
              w.z = pack_bf16(__uint_as_float(r[v4 * 8 + 4]) * inv, __uint_as_float(r[v4 * 8 + 5]) * inv);
              w.w = pack_bf16(__uint_as_float(r[v4 * 8 + 6]) * inv, __uint_as_float(r[v4 * 8 + 7]) * inv);
              dst[v4] = w;
            }
          }
        }
        if (valid) p.lse[orow] = denom > 0.f ? (msub + log2f(denom)) * LN2 : -INFINITY;
      } else {
        const int64_t prow = static_cast<int64_t>(split) * p.B * p.T * p.H + orow;
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
        for (int c4 = 0; c4 < C / 32; ++c4) {
          uint32_t r[32];
          if (ntiles > 0) {
            tmem_ld32(tO + c4 * 32, r);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = 0u;
          }
          if (valid) {
            float4* dst = reinterpret_cast<float4*>(p.part_o + prow * C + c4 * 32);
#pragma unroll
            for (int v4 = 0; v4 < 8; ++v4)
              dst[v4] = make_float4(__uint_as_float(r[v4 * 4]) * inv, __uint_as_float(r[v4 * 4 + 1]) * inv,
                                    __uint_as_float(r[v4 * 4 + 2]) * inv, __uint_as_float(r[v4 * 4 + 3]) * inv);
          }
        }
        if (valid) p.part_lse[prow] = l > 0.f ? (msub + log2f(l)) * LN2 : -INFINITY;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace wpt
