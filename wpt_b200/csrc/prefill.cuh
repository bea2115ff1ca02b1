// Prefill / verification attention forward for one key-value head (MQA),
// tcgen05 + TMEM + TMA on sm_100a.
//
// Computes WPT's exact_attention output and log-sum-exp
// (packages/wpt-model/src/wpt_model/pytorch_kernels.py:98-121) for many
// queries per row, the window/sink form (pytorch_kernels.py:171-187 over a
// contiguous window; attention.py:85-107) and tree-masked verification.
//
// Tiles. A work item is BM = 128 "rows": TQ = 128 / H consecutive query
// tokens of one batch row, each with its H heads (row r = token r / H, head
// r % H). All heads of MQA read the same keys, so one K/V tile serves every
// row, and the 128 rows are the M of both products:
//   S  = Q K^T   M=128 rows, N=128 keys, K=C    A=Q (smem), B=K (smem)
//   O += P V     M=128 rows, N=C,       K=128  A=P (TMEM),  B=V (smem, MN-major)
//
// Persistent schedule. One CTA per SM walks the work items (query tile,
// batch row, key split) from the most expensive (the last query tiles) down,
// item c, c + gridDim.x, ... The loader keeps prefetching across item
// boundaries: Q has QB shared-memory buffers, and K and V stream through
// separate rings (KST and VST stages) so a K stage is released as soon as
// its S product completes and a V stage once its P V product does. TMEM
// holds S twice (2 x 128 columns, one per key tile in flight) and O twice
// (one per item in flight, 2 x C columns), so an item's epilogue overlaps
// the next item's products. P (bf16) overwrites the first 64 columns of its
// S buffer.
//
// Warps: 4 x SLICES softmax warps, then the tcgen05 issuer (one lane) and the
// TMA loader (one lane). Warp w reads TMEM lane quadrant w % 4 (rows
// 32 (w % 4) ..), so SLICES warps share each quadrant: each thread owns one
// row and a slice of 128 / SLICES of its keys. The slices of a row exchange
// their maxima through shared memory once per tile and all take the same
// lazy-maximum decision; each rescales and writes its slice of O.
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
// Key slices wholly inside a row's range skip the per-element mask.
//
// Split-KV: an item's key tiles may be split; with splits > 1 each split
// writes its normalised partial output and LSE (no sink) for the merge
// kernel, which adds the sink.
//
// Barrier phases run on across items: key tile g (counted over the CTA's
// items) uses K stage g % KST, V stage g % VST and S buffer g % 2; the n-th
// item with any key tile uses Q buffer n % QB and O buffer n % 2.
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
  int B, T, H, N, window, TQ, splits, items;
  float scale_log2;  // softmax scale * log2(e)
};

template <int C, int QB, int KST, int VST, int SLICES>
struct PrefillLayout {
  static constexpr int BM = 128, BN = 128;
  static constexpr int SUB = C / 64;  // 64-element (128-byte) column chunks
  static constexpr int Q_BYTES = BM * C * 2;
  static constexpr int KV_BYTES = BN * C * 2;  // one K or V tile
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = QB * Q_BYTES;
  static constexpr int OFF_V = OFF_K + KST * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + VST * KV_BYTES;
  // q_full[QB], q_empty[QB], k_full[KST], k_empty[KST], v_full[VST], v_empty[VST],
  // s_full[2], p_ready[2], o_done, o_final[2], o_free[2]
  static constexpr int NBAR = 2 * QB + 2 * KST + 2 * VST + 4 + 1 + 4;
  // row maxima for two tiles, then row sums: (3, SLICES, 128) floats
  static constexpr int OFF_RED = OFF_BAR + NBAR * 8;
  static constexpr int OFF_MISC = OFF_RED + 3 * SLICES * 128 * 4;
  static constexpr int BYTES = OFF_MISC + 16 + 1024;  // + slack to align the base to 1024
  static constexpr int THREADS = 32 * (4 * SLICES + 2);
  static constexpr int MMA_WARP = 4 * SLICES, LOAD_WARP = 4 * SLICES + 1;
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

// Work item k: the most expensive query tiles first, then batch row, then split.
struct PrefillItem {
  int b, t0, split, tile0, ntiles;
};

// Called by all 32 lanes of a warp: lane i reads the positions of tokens
// t0 + i, t0 + i + 32, ... and warp reductions give the item's key range,
// one global-load round trip for the usual TQ <= 32.
__device__ __forceinline__ PrefillItem prefill_item(const PrefillParams& p, int k) {
  PrefillItem it;
  const int lane = threadIdx.x & 31;
  const int per_tile = p.B * p.splits;
  const int nq = (p.T + p.TQ - 1) / p.TQ;
  const int qtile = nq - 1 - k / per_tile;
  const int rem = k - (k / per_tile) * per_tile;
  it.b = rem / p.splits;
  it.split = rem - it.b * p.splits;
  it.t0 = qtile * p.TQ;
  int row_lo = INT_MAX, row_hi = -1;
  const int tq_end = min(p.TQ, p.T - it.t0);
  for (int tq = lane; tq < tq_end; tq += 32) {
    int lo, hi;
    prefill_query_rows(p, it.b, it.t0 + tq, lo, hi);
    if (hi >= lo) {
      row_lo = min(row_lo, lo);
      row_hi = max(row_hi, hi);
    }
  }
  row_lo = __reduce_min_sync(0xffffffffu, row_lo);
  row_hi = __reduce_max_sync(0xffffffffu, row_hi);
  it.tile0 = 0;
  it.ntiles = 0;
  if (row_hi >= row_lo) {
    const int first = row_lo / 128, last = row_hi / 128, total = last - first + 1;
    const int per = (total + p.splits - 1) / p.splits;
    it.tile0 = first + it.split * per;
    const int left = last + 1 - it.tile0;
    it.ntiles = left < per ? (left > 0 ? left : 0) : per;
  }
  return it;
}

// N consecutive TMEM columns of this warp's lanes into registers (one wait).
template <int N>
__device__ __forceinline__ void tmem_cols(uint32_t taddr, uint32_t (&r)[N]) {
  if constexpr (N == 128) {
    tmem_ld128(taddr, r);
  } else if constexpr (N == 64) {
    tmem_ld64(taddr, r);
  } else if constexpr (N == 32) {
    tmem_ld32(taddr, r);
  } else {
    static_assert(N == 16, "16, 32, 64 or 128 columns");
    tmem_ld16(taddr, r);
  }
}

template <int C, int QB, int KST, int VST, int SLICES>
__global__ void __launch_bounds__(PrefillLayout<C, QB, KST, VST, SLICES>::THREADS, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const PrefillParams p) {
  using L = PrefillLayout<C, QB, KST, VST, SLICES>;
  constexpr int BM = L::BM, BN = L::BN, SUB = L::SUB;
  constexpr int KS = BN / SLICES;  // keys per softmax thread
  constexpr int OS = C / SLICES;   // output columns per softmax thread
  constexpr int NSOFT = 128 * SLICES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + QB;
  uint64_t* k_full = q_empty + QB;
  uint64_t* k_empty = k_full + KST;
  uint64_t* v_full = k_empty + KST;
  uint64_t* v_empty = v_full + VST;
  uint64_t* s_full = v_empty + VST;
  uint64_t* p_ready = s_full + 2;
  uint64_t* o_done = p_ready + 2;  // one phase per P V product
  uint64_t* o_final = o_done + 1;  // [O buffer]: one phase per item, after its last P V
  uint64_t* o_free = o_final + 2;  // [O buffer]: the epilogue has read it
  float* s_red = reinterpret_cast<float*>(smem + L::OFF_RED);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < QB; ++s) {
      mbar_init(q_full + s, 1);
      mbar_init(q_empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(s_full + s, 1);
      mbar_init(p_ready + s, NSOFT);
      mbar_init(o_final + s, 1);
      mbar_init(o_free + s, NSOFT);
    }
    for (int s = 0; s < KST; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(k_empty + s, 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(v_full + s, 1);
      mbar_init(v_empty + s, 1);
    }
    mbar_init(o_done, 1);
    fence_mbar_init();
  }
  if (warp == L::MMA_WARP) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  if (warp == L::LOAD_WARP && lane == 0) {
    tma_prefetch(&tm_q);
    tma_prefetch(&tm_k);
    tma_prefetch(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;  // S buffers at columns 0 and 128, O buffers at 256 and 256 + C

  if (warp == L::LOAD_WARP) {
    // ------------------------------------------------------------ TMA loader
    bool ok = true;
    int g = 0, n = 0;  // key tiles issued so far, items with key tiles so far
    for (int k = blockIdx.x; ok && k < p.items; k += gridDim.x) {
      const PrefillItem it = prefill_item(p, k);  // the whole warp
      if (it.ntiles == 0) continue;
      if (lane == 0) {
        const int qb = n % QB;
        if (n >= QB) ok = mbar_wait(q_empty + qb, ((n / QB) & 1) ^ 1, p.status);
        if (ok) {
          mbar_expect_tx(q_full + qb, L::Q_BYTES);
          const int qrow0 = (it.b * p.T + it.t0) * p.H;
          for (int s = 0; s < SUB; ++s)
            tma_load_2d(sQ + qb * L::Q_BYTES + s * BM * 128, &tm_q, q_full + qb, s * 64, qrow0);
        }
        for (int j = 0; ok && j < it.ntiles; ++j) {
          const int gg = g + j, n0 = (it.tile0 + j) * BN;
          const int ks = gg % KST, vs = gg % VST;
          if (gg >= KST && !(ok = mbar_wait(k_empty + ks, ((gg / KST) & 1) ^ 1, p.status))) break;
          mbar_expect_tx(k_full + ks, L::KV_BYTES);
          for (int s = 0; s < SUB; ++s)
            tma_load_3d(sK + ks * L::KV_BYTES + s * BN * 128, &tm_k, k_full + ks, s * 64, n0, it.b);
          if (gg >= VST && !(ok = mbar_wait(v_empty + vs, ((gg / VST) & 1) ^ 1, p.status))) break;
          mbar_expect_tx(v_full + vs, L::KV_BYTES);
          for (int s = 0; s < SUB; ++s)
            tma_load_3d(sV + vs * L::KV_BYTES + s * BN * 128, &tm_v, v_full + vs, s * 64, n0, it.b);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      g += it.ntiles;
      ++n;
    }
    // the consumers wait for every copy issued here before the CTA leaves
    // (or time out together with this thread), so nothing lands after exit
  } else if (warp == L::MMA_WARP) {
    // ------------------------------------------------------ tcgen05 issuer
    constexpr uint32_t IDESC_S = idesc_bf16(BM, BN, 0, 0);
    constexpr uint32_t IDESC_O = idesc_bf16(BM, C, 0, 1);
    const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
    bool ok = true;
    int g = 0, n = 0;
    for (int k = blockIdx.x; ok && k < p.items; k += gridDim.x) {
      const PrefillItem it = prefill_item(p, k);  // the whole warp
      if (it.ntiles == 0) continue;
      if (lane == 0) {
        const int qb = n % QB, ob = n & 1;
        const uint32_t tO = tmem + 256 + ob * C;
        ok = mbar_wait(q_full + qb, (n / QB) & 1, p.status);
        if (ok && n >= 2) ok = mbar_wait(o_free + ob, ((n >> 1) & 1) ^ 1, p.status);
        for (int j = 0; ok && j <= it.ntiles; ++j) {
          if (j < it.ntiles) {  // S(g + j) = Q K^T
            const int gs = g + j, ks = gs % KST;
            if (!(ok = mbar_wait(k_full + ks, (gs / KST) & 1, p.status))) break;
            tc_fence_after();
            const uint32_t d = tmem + (gs & 1) * 128;
#pragma unroll
            for (int kk = 0; kk < C / 16; ++kk) {
              const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
              mma_ss(d, sdesc_sw128(q_addr + qb * L::Q_BYTES + off, 16, 1024),
                     sdesc_sw128(k_addr + ks * L::KV_BYTES + off, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
            }
            mma_commit(k_empty + ks);
            mma_commit(s_full + (gs & 1));
            if (j == it.ntiles - 1) mma_commit(q_empty + qb);  // the item's last reader of Q
          }
          if (j > 0) {  // O += P V for key tile g + j - 1
            const int gp = g + j - 1, vs = gp % VST;
            if (!(ok = mbar_wait(p_ready + (gp & 1), (gp >> 1) & 1, p.status))) break;
            if (!(ok = mbar_wait(v_full + vs, (gp / VST) & 1, p.status))) break;
            tc_fence_after();
            const uint32_t a = tmem + (gp & 1) * 128;
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk) {
              mma_ts(tO, a + kk * 8, sdesc_sw128(v_addr + vs * L::KV_BYTES + kk * 16 * 128, BN * 128, 1024), IDESC_O,
                     (j > 1 || kk > 0) ? 1u : 0u);
            }
            mma_commit(v_empty + vs);
            mma_commit(o_done);
            if (j == it.ntiles) mma_commit(o_final + ob);
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      g += it.ntiles;
      ++n;
    }
  } else {
    // ---------------- softmax: one row and a slice of its keys per thread
    const int quad = warp & 3, slice = warp >> 2;
    const int row = quad * 32 + lane;
    const int tq = row / p.H, h = row - tq * p.H;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float sl2 = p.scale_log2;
    const int64_t rows_all = static_cast<int64_t>(p.B) * p.T * p.H;
    bool ok = true;
    int g = 0, n = 0;
    for (int k = blockIdx.x; ok && k < p.items; k += gridDim.x) {
      const PrefillItem it = prefill_item(p, k);
      const int t = it.t0 + tq;
      const bool valid = tq < p.TQ && t < p.T;
      const int64_t orow = (static_cast<int64_t>(it.b) * p.T + t) * p.H + h;
      if (it.ntiles == 0) {  // an empty split: nothing to read
        if (valid && slice == 0) {
          if (p.splits > 1) {
            p.part_lse[static_cast<int64_t>(it.split) * rows_all + orow] = -INFINITY;
          } else {
            for (int c = 0; c < C; ++c) p.out[orow * C + c] = __float2bfloat16_rn(0.f);
            p.lse[orow] = p.sink != nullptr ? p.sink[h] : -INFINITY;
          }
        }
        continue;
      }
      const int ob = n & 1;
      const uint32_t tO = lane_addr + 256 + ob * C + slice * OS;
      int lo = 0, hi = -1;
      if (valid) prefill_query_rows(p, it.b, t, lo, hi);
      int64_t tbase = int64_t(1) << 62;  // no tree: a base no row reaches
      uint64_t tbits = ~0ull;
      if (valid && p.tree_bits) {
        tbase = p.tree_base[it.b];
        tbits = p.tree_bits[static_cast<int64_t>(it.b) * p.T + t];
      }
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < it.ntiles; ++j) {
        const int gs = g + j;
        ok = __all_sync(0xffffffffu, mbar_wait(s_full + (gs & 1), (gs >> 1) & 1, p.status));
        if (!ok) break;
        tc_fence_after();
        const int n0 = (it.tile0 + j) * BN + slice * KS;  // this thread's first key
        const uint32_t sAddr = lane_addr + (gs & 1) * 128;
        uint32_t r[KS];
        tmem_cols<KS>(sAddr + slice * KS, r);
        const bool whole = valid && n0 >= lo && n0 + KS - 1 <= hi &&
                           (static_cast<int64_t>(n0) + KS - 1 < tbase || static_cast<int64_t>(n0) >= tbase + 64);
        float tmax = -INFINITY;
        if (whole) {
#pragma unroll
          for (int i = 0; i < KS; ++i) tmax = fmaxf(tmax, __uint_as_float(r[i]));
        } else {
#pragma unroll
          for (int i = 0; i < KS; ++i) {
            const int nn = n0 + i;
            bool vis = valid && nn >= lo && nn <= hi;
            const int64_t d = static_cast<int64_t>(nn) - tbase;
            if (d >= 0 && d < 64) vis = vis && ((tbits >> d) & 1ull);
            if (!vis) r[i] = __float_as_uint(-INFINITY);
            tmax = fmaxf(tmax, __uint_as_float(r[i]));
          }
        }
        if constexpr (SLICES > 1) {  // the row's maximum over its slices (double-buffered by tile parity)
          float* red = s_red + (gs & 1) * SLICES * 128;
          red[slice * 128 + row] = tmax;
          named_barrier(1, NSOFT);
#pragma unroll
          for (int o = 0; o < SLICES; ++o)
            if (o != slice) tmax = fmaxf(tmax, red[o * 128 + row]);
        }
        tmax *= sl2;
        const bool need = tmax > m_used + 8.f;
        const float alpha = need ? fast_exp2(m_used - tmax) : 1.f;
        if (__any_sync(0xffffffffu, need) && j > 0) {  // every slice's warp votes alike: same rows, same maxima
          ok = __all_sync(0xffffffffu, mbar_wait(o_done, (gs - 1) & 1, p.status));
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < OS; c += 16) {
            uint32_t o[16];
            tmem_ld16(tO + c, o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st16(tO + c, o);
          }
        }
        if (need) {
          l *= alpha;
          m_used = tmax;
        }
        const float msub = m_used == -INFINITY ? 0.f : m_used;
        // the weights of this slice as bf16 pairs, over columns [slice KS / 2, (slice + 1) KS / 2) of S
#pragma unroll
        for (int c = 0; c < KS / 2; c += 32 < KS / 2 ? 32 : KS / 2) {
          constexpr int NP = 32 < KS / 2 ? 32 : KS / 2;
          uint32_t pk[NP];
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            const float e0 = fast_exp2(fmaf(__uint_as_float(r[2 * (c + i)]), sl2, -msub));
            const float e1 = fast_exp2(fmaf(__uint_as_float(r[2 * (c + i) + 1]), sl2, -msub));
            l += e0 + e1;
            pk[i] = pack_bf16(e0, e1);
          }
          if constexpr (NP == 32) {
            tmem_st32(sAddr + slice * (KS / 2) + c, pk);
          } else {
            tmem_st16(sAddr + slice * (KS / 2) + c, pk);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(p_ready + (gs & 1));
      }
      if (!ok) break;
      // o_done's parity cannot name the item's last product (the MMA may still
      // be two products behind), so the epilogue waits on o_final, which
      // completes once per item and O buffer, after the item's last product
      ok = __all_sync(0xffffffffu, mbar_wait(o_final + ob, (n >> 1) & 1, p.status));
      if (!ok) break;
      tc_fence_after();
      if constexpr (SLICES > 1) {  // the row's sum over its slices
        float* lred = s_red + 2 * SLICES * 128;
        lred[slice * 128 + row] = l;
        named_barrier(1, NSOFT);
        l = 0.f;
#pragma unroll
        for (int o = 0; o < SLICES; ++o) l += lred[o * 128 + row];
      }
      const float msub = m_used == -INFINITY ? 0.f : m_used;
      float denom = l;
      if (p.splits == 1 && p.sink != nullptr && valid) denom += fast_exp2(fmaf(p.sink[h], LOG2E, -msub));
      const float inv = denom > 0.f ? 1.f / denom : 0.f;
#pragma unroll
      for (int c = 0; c < OS; c += 16) {
        uint32_t o16[16];
        tmem_ld16(tO + c, o16);
        if (!valid) continue;
        if (p.splits == 1) {
          uint4* dst = reinterpret_cast<uint4*>(p.out + orow * C + slice * OS + c);
#pragma unroll
          for (int v4 = 0; v4 < 2; ++v4) {
            uint4 w;
            w.x = pack_bf16(__uint_as_float(o16[v4 * 8 + 0]) * inv, __uint_as_float(o16[v4 * 8 + 1]) * inv);
            w.y = pack_bf16(__uint_as_float(o16[v4 * 8 + 2]) * inv, __uint_as_float(o16[v4 * 8 + 3]) * inv);
            w.z = pack_bf16(__uint_as_float(o16[v4 * 8 + 4]) * inv, __uint_as_float(o16[v4 * 8 + 5]) * inv);
            w.w = pack_bf16(__uint_as_float(o16[v4 * 8 + 6]) * inv, __uint_as_float(o16[v4 * 8 + 7]) * inv);
            dst[v4] = w;
          }
        } else {
          const int64_t prow = static_cast<int64_t>(it.split) * rows_all + orow;
          float4* dst = reinterpret_cast<float4*>(p.part_o + prow * C + slice * OS + c);
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4)
            dst[v4] = make_float4(__uint_as_float(o16[v4 * 4]) * inv, __uint_as_float(o16[v4 * 4 + 1]) * inv,
                                  __uint_as_float(o16[v4 * 4 + 2]) * inv, __uint_as_float(o16[v4 * 4 + 3]) * inv);
        }
      }
      tc_fence_before();
      mbar_arrive(o_free + ob);  // O buffer ob may be overwritten by the item after next
      if (valid && slice == 0) {
        if (p.splits == 1) {
          p.lse[orow] = denom > 0.f ? (msub + log2f(denom)) * LN2 : -INFINITY;
        } else {
          p.part_lse[static_cast<int64_t>(it.split) * rows_all + orow] =
              l > 0.f ? (msub + log2f(l)) * LN2 : -INFINITY;
        }
      }
      g += it.ntiles;
      ++n;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == L::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace wpt
