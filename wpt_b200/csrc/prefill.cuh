// Prefill / verification attention forward for one key-value head (MQA),
// tcgen05 + TMEM + TMA on sm_100a.
//
// Computes WPT's exact_attention output and log-sum-exp
// (packages/wpt-model/src/wpt_model/pytorch_kernels.py:98-121) for many
// queries per row, the window/sink form (pytorch_kernels.py:171-187 over a
// contiguous window; attention.py:85-107) and tree-masked verification.
//
// Tiles. A query tile is BM = 128 "rows": TQ = 128 / H consecutive query
// tokens of one batch row, each with its H heads (row r = token r / H, head
// r % H). All heads of MQA read the same keys, so one K/V tile serves every
// row, and the 128 rows are the M of both products:
//   S  = Q K^T   M=128 rows, N=128 keys, K=C    A=Q (smem), B=K (smem)
//   O += P V     M=128 rows, N=C,       K=128  A=P (TMEM),  B=V (smem, MN-major)
// A work item is a pair of consecutive query tiles, A (tokens t0 ..) and B
// (tokens t0 + TQ ..), of one batch row and key split: both read the same
// key tiles, so each K and V tile is loaded once for 256 rows.
//
// Warps. Softmax warpgroup A (warps 0-3) owns tile A, warpgroup B (warps
// 4-7) tile B: warp w reads TMEM lane quadrant w % 4 and each thread owns
// one row and all 128 keys of a key tile, so no thread exchanges anything
// with another. Warp 8 issues the tcgen05 products (one lane), warp 9 runs
// the TMA loads (one lane) and publishes each item's key-tile range to the
// other warps through a small shared-memory ring.
//
// Pipeline. TMEM holds S_A, S_B (128 columns each, P as bf16 pairs over the
// first 64 columns of its S) and O_A, O_B (C columns each). Per key tile j
// the issuer runs PV_A(j-1), S_A(j), PV_B(j-1), S_B(j): while warpgroup A
// turns S_A(j) into P the tensor pipe works on B's products and the other
// way round. tcgen05 products of one thread run in issue order, so S_A(j)
// overwrites P_A(j-1) only after PV_A(j-1) has read it, and the commit that
// says S_A(j) is ready also says PV_A(j-1) is done, which is what a rescale
// of O_A needs. Q pairs have QB buffers; K and V tiles stream through one
// ring of NS stages, K one tile ahead: K(0), K(1), V(0), K(2), V(1), ...
//
// Output: a full query tile's rows go, as bf16, into the item's own Q
// buffer (free once the item's last product is done) in the swizzled
// layout of a TMA box, and one TMA store per 64 columns writes them out; the
// loader reloads that buffer only after the store has read it (q_stored).
//
// Online softmax in base 2 with a lazy maximum: a row's running maximum is
// only raised (and O rescaled) when a tile's maximum exceeds it by more
// than 8, so P stays below 2^8 and O is rarely touched. The rescale is done
// by every lane of a warp when any lane needs it (tcgen05.ld/st are
// warp-collective). P is handed to the issuer in two halves of 64 keys
// (p_half, then p_ready), so the first half of P V runs while the second
// half of P is computed. Exponentials: POLY8 of every 8 pairs of weights
// are computed on the FMA pipe (exp2_poly_pair), the rest with ex2.approx,
// so the two pipes share the work.
//
// Masks. Query t at position p (its own table row) reads rows lo..hi:
//   hi = min(p, N - 1); lo = max(0, p - window + 1 when window > 0, floor[b,t]).
// Tree mode adds: rows tree_base[b] + i (0 <= i < 64) are visible only when
// bit i of tree_bits[b, t] is set (node t sees itself and its ancestors).
// Key tiles wholly inside a row's range skip the per-element mask.
//
// Split-KV: an item's key tiles may be split; with splits > 1 each split
// writes its normalised partial output and LSE (no sink) for the merge
// kernel, which adds the sink. Cluster mode (2 splits, one item per CTA):
// the two splits of a pair are one 2-CTA cluster; each CTA leaves its
// partials in its idle K/V ring and, after a cluster barrier, the CTA of
// rank w combines query tile w's rows from both (distributed shared memory)
// with the sink, so no partials go to HBM and no merge kernel runs.
//
// Barrier phases run on across items: key tile g (counted over the CTA's
// items) is ring entries prefill_k_entry(g) (K) and prefill_v_entry(g) (V);
// the n-th item with any key tile uses Q buffer n % QB; the idx-th item of
// the CTA uses ring slot idx % IR of the item ring.
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
  int tma_out;       // 1: full query tiles leave through shared memory and a TMA store (tm_o)
  int cluster;       // 1: splits == 2, one item per CTA, a pair's two splits one 2-CTA cluster that
                     // combines them in shared memory (no partials in HBM, no merge launch); the
                     // kernel's CLUSTER instance
  float scale_log2;  // softmax scale * log2(e)
};

template <int C, int QB, int NS>
struct PrefillLayout {
  static constexpr int BM = 128, BN = 128;
  static constexpr int SUB = C / 64;           // 64-element (128-byte) column chunks
  static constexpr int QT_BYTES = BM * C * 2;  // one query tile
  static constexpr int Q_BYTES = 2 * QT_BYTES; // a pair
  static constexpr int KV_BYTES = BN * C * 2;  // one K or V tile
  static constexpr int IR = 4;                 // item ring slots
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = QB * Q_BYTES;
  static constexpr int OFF_BAR = OFF_KV + NS * KV_BYTES;
  // q_full[QB], q_empty[QB], kv_full[NS], kv_empty[NS], s_full[2], p_half[2],
  // p_ready[2], o_final[2], o_free[2], item_full[IR], item_empty[IR], q_stored[QB]
  static constexpr int NBAR = 3 * QB + 2 * NS + 10 + 2 * IR;
  static constexpr int OFF_ITEM = OFF_BAR + NBAR * 8;  // IR x (first key tile, key tiles)
  static constexpr int OFF_MISC = OFF_ITEM + IR * 8;
  static constexpr int BYTES = OFF_MISC + 16 + 1024;  // + slack to align the base to 1024
  // warpgroups 0 and 1: softmax; warpgroup 2: the issuer, the loader and two idle warps
  static constexpr int THREADS = 384;
  static constexpr int MMA_WARP = 8, LOAD_WARP = 9;
  // registers per thread after setmaxnreg: 168 at launch (65536 / 384), then
  // 128 x 56 + 256 x 224 = 384 x 168, the block's whole allocation
  static constexpr int REGS_LAUNCH = 168, REGS_CONTROL = 56, REGS_SOFTMAX = 224;
  static_assert(128 * REGS_CONTROL + 256 * REGS_SOFTMAX == THREADS * REGS_LAUNCH, "register split");
  static constexpr int ITEM_READERS = 9;  // the issuer warp and the 8 softmax warps
  // cluster mode: each query tile's normalised partial, (C / 4) x 128 rows of
  // float4 then 128 log-sums, in the K/V ring (idle once the item's last
  // product is done)
  static constexpr int STASH_BYTES = C * 128 * 4 + 128 * 4;
  static_assert(2 * STASH_BYTES <= NS * KV_BYTES, "cluster stash exceeds the K/V ring");
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

// Work item k: the most expensive query-tile pairs first, then batch row, then split.
struct PrefillItem {
  int b, t0, split, tile0, ntiles;
};

__device__ __forceinline__ PrefillItem prefill_place(const PrefillParams& p, int k) {
  PrefillItem it;
  const int per_pair = p.B * p.splits;
  const int np = (p.T + 2 * p.TQ - 1) / (2 * p.TQ);
  const int qpair = np - 1 - k / per_pair;
  const int rem = k - (k / per_pair) * per_pair;
  it.b = rem / p.splits;
  it.split = rem - it.b * p.splits;
  it.t0 = qpair * 2 * p.TQ;
  it.tile0 = 0;
  it.ntiles = 0;
  return it;
}

// The key tiles of item k. Called by all 32 lanes of a warp: lane i reads
// the positions of tokens t0 + i, t0 + i + 32, ... and warp reductions give
// the pair's key range.
__device__ __forceinline__ PrefillItem prefill_item(const PrefillParams& p, int k) {
  PrefillItem it = prefill_place(p, k);
  const int lane = threadIdx.x & 31;
  int row_lo = INT_MAX, row_hi = -1;
  const int tq_end = min(2 * p.TQ, p.T - it.t0);
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
  if (row_hi >= row_lo) {
    const int first = row_lo / 128, last = row_hi / 128, total = last - first + 1;
    const int per = (total + p.splits - 1) / p.splits;
    it.tile0 = first + it.split * per;
    const int left = last + 1 - it.tile0;
    it.ntiles = left < per ? (left > 0 ? left : 0) : per;
  }
  return it;
}

// Visibility of 32 consecutive tile columns (bit i: column c0 + i) for a
// row that sees columns a..b (relative to c0) and, in a tree tile, only the
// tree rows whose bits are set: sh is the tree-bit index of column c0.
__device__ __forceinline__ uint32_t prefill_visible_word(int a, int b, bool in_tree, int sh, uint64_t tbits) {
  const int lo = a < 0 ? 0 : (a > 32 ? 32 : a);
  const int hi = b < -1 ? 0 : (b >= 31 ? 32 : b + 1);  // columns lo .. hi - 1
  uint32_t m = hi <= lo ? 0u : ((hi == 32 ? 0xFFFFFFFFu : ((1u << hi) - 1u)) & ~((1u << lo) - 1u));
  if (in_tree && sh > -32 && sh < 64) {
    uint32_t t;  // tree bits of the columns inside the tree, ones outside it
    if (sh >= 0) {
      t = static_cast<uint32_t>(tbits >> sh);
      if (sh > 32) t |= 0xFFFFFFFFu << (64 - sh);
    } else {
      t = (static_cast<uint32_t>(tbits) << -sh) | ((1u << -sh) - 1u);
    }
    m &= t;
  }
  return m;
}

// Ring entries of key tile g (counted over the CTA's items): the loader
// runs K one tile ahead of V, K(0) K(1) V(0) K(2) V(1) ..., which gives
// each K load about two and a half rounds of the issue loop before it is
// read and each V load one and a half. Entry 2G - 1 (a K(G) after the last
// tile) is never used.
__device__ __forceinline__ int prefill_k_entry(int g) { return g == 0 ? 0 : 2 * g - 1; }
__device__ __forceinline__ int prefill_v_entry(int g) { return 2 * g + 2; }

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Weights of 64 scores (one half of a row's key tile) as 32 bf16 pairs
// against msub, their fp32 sum, and (rmax) the maximum of s * sl2 - msub
// over them, found in the same pass.
template <int POLY8>
__device__ __forceinline__ float prefill_half_weights(const uint32_t (&r)[64], float sl2, float msub,
                                                      uint32_t (&pk)[32], float& rmax) {
  const uint64_t s2 = f2_pack(sl2, sl2), nm = f2_pack(-msub, -msub);
  uint64_t acc[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
  float m[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const uint64_t x = f2_fma(f2_pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), s2, nm);
    float x0, x1, e0, e1;
    f2_unpack(x, x0, x1);
    m[i & 1] = max3f(m[i & 1], x0, x1);
    if ((i & 7) < POLY8) {
      exp2_poly_pair(x0, x1, e0, e1);
    } else {
      e0 = fast_exp2(x0);
      e1 = fast_exp2(x1);
    }
    pk[i] = pack_bf16(e0, e1);
    acc[i & 1] = f2_add(acc[i & 1], f2_pack(e0, e1));
  }
  rmax = fmaxf(m[0], m[1]);
  float a0, a1, b0, b1;
  f2_unpack(acc[0], a0, a1);
  f2_unpack(acc[1], b0, b1);
  return (a0 + a1) + (b0 + b1);
}

// Maximum of 128 values as a tree of three-input maxima (depth 5: 43, 15,
// 5, 2, 1 nodes), so the latency is a few instructions, not a chain.
__device__ __forceinline__ float max128(const uint32_t (&r)[128]) {
  float a[43];
#pragma unroll
  for (int i = 0; i < 42; ++i)
    a[i] = max3f(__uint_as_float(r[3 * i]), __uint_as_float(r[3 * i + 1]), __uint_as_float(r[3 * i + 2]));
  a[42] = fmaxf(__uint_as_float(r[126]), __uint_as_float(r[127]));
  float b[15];
#pragma unroll
  for (int i = 0; i < 14; ++i) b[i] = max3f(a[3 * i], a[3 * i + 1], a[3 * i + 2]);
  b[14] = a[42];
  float c[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) c[i] = max3f(b[3 * i], b[3 * i + 1], b[3 * i + 2]);
  return max3f(max3f(c[0], c[1], c[2]), c[3], c[4]);
}

// Multiplies this warp's rows of O (C TMEM columns from oAddr) by alpha.
template <int C>
__device__ __forceinline__ void prefill_rescale_o(uint32_t oAddr, float alpha) {
#pragma unroll
  for (int c = 0; c < C; c += 32) {
    uint32_t o[32];
    tmem_ld32(oAddr + c, o);
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
    tmem_st32(oAddr + c, o);
  }
}

// Sets the scores of the tile columns c0 .. c0 + 63 this row may not read
// to -inf (a, b: the row's visible tile columns; tb: the tree's first tile
// column).
__device__ __forceinline__ void prefill_mask_half(uint32_t (&r)[64], int c0, int a, int b, bool in_tree, int tb,
                                                  uint64_t tbits) {
#pragma unroll
  for (int wd = 0; wd < 2; ++wd) {
    const int cw = c0 + 32 * wd;
    const uint32_t vis = prefill_visible_word(a - cw, b - cw, in_tree, cw - tb, tbits);
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (!((vis >> i) & 1u)) r[32 * wd + i] = __float_as_uint(-INFINITY);
  }
}

// S_w = Q_w K^T for key tile gs into S buffer w (TMEM column 128 w), then
// a commit on s_full[w]. qa: the Q pair's shared-memory address. Called by
// the whole issuer warp (one elected lane issues): each descriptor is a
// warp-uniform base plus a constant offset (addresses are in 16-byte units
// in the low 14 bits, and no shared-memory address carries out of them).
template <int KK>
__device__ __forceinline__ void prefill_s_steps(uint32_t d, uint64_t dq, uint64_t dk, uint32_t idesc) {
  if constexpr (KK > 0) prefill_s_steps<KK - 1>(d, dq, dk, idesc);
  constexpr uint32_t off = ((KK >> 2) * (128 * 128) + (KK & 3) * 32) >> 4;
  mma_ss_off_warp<off, off>(d, dq, dk, idesc, KK > 0 ? 1u : 0u);
}
template <int C, int NS, int QT_BYTES, int KV_BYTES>
__device__ __forceinline__ void prefill_issue_s(uint32_t tmem, uint32_t qa, uint32_t kv_addr, int w, int gs,
                                                uint64_t* s_full) {
  const uint64_t dq = sdesc_sw128(qa + w * QT_BYTES, 16, 1024);
  const uint64_t dk = sdesc_sw128(kv_addr + (prefill_k_entry(gs) % NS) * KV_BYTES, 16, 1024);
  prefill_s_steps<C / 16 - 1>(tmem + w * 128, dq, dk, idesc_bf16(128, 128, 0, 0));
  mma_commit_warp(s_full + w);
}

// O_w += P_w V for key tile gp over its keys 64 HALF .. 64 HALF + 63 (first:
// O_w = P_w V). P_w is bf16 pairs over the first 64 columns of S buffer w;
// V is MN-major in its ring stage.
template <int KK, int KK0>
__device__ __forceinline__ void prefill_pv_steps(uint32_t d, uint32_t a, uint64_t dv, uint32_t idesc, uint32_t acc0) {
  if constexpr (KK > KK0) prefill_pv_steps<KK - 1, KK0>(d, a, dv, idesc, acc0);
  constexpr uint32_t off = (KK * 16 * 128) >> 4;
  mma_ts_off_warp<KK * 8, off>(d, a, dv, idesc, KK > 0 ? 1u : acc0);
}
template <int C, int NS, int KV_BYTES, int HALF>
__device__ __forceinline__ void prefill_issue_pv(uint32_t tmem, uint32_t kv_addr, int w, int gp, bool first) {
  const uint64_t dv = sdesc_sw128(kv_addr + (prefill_v_entry(gp) % NS) * KV_BYTES, 128 * 128, 1024);
  prefill_pv_steps<4 * HALF + 3, 4 * HALF>(tmem + 256 + w * C, tmem + w * 128, dv, idesc_bf16(128, C, 0, 1),
                                           first ? 0u : 1u);
}

// Cluster mode, after the item: the rows of query tile `w` (= this CTA's
// rank in the pair's cluster) from this CTA's stash and its partner's
// (distributed shared memory), with the sink: out and lse of those rows.
template <int C, int STASH_BYTES>
__device__ __forceinline__ void prefill_cluster_combine(const PrefillParams& p, uint8_t* sKV, int w, int row) {
  const PrefillItem it = prefill_place(p, blockIdx.x);
  const int tq = row / p.H, h = row - tq * p.H;
  const int t = it.t0 + w * p.TQ + tq;
  if (tq >= p.TQ || t >= p.T) return;
  const int64_t orow = (static_cast<int64_t>(it.b) * p.T + t) * p.H + h;
  const uint32_t mine = smem_u32(sKV) + w * STASH_BYTES;
  const uint32_t theirs = dsmem_map(mine, static_cast<uint32_t>(w ^ 1));
  const float* own = reinterpret_cast<const float*>(sKV + w * STASH_BYTES);
  const float l0 = own[C * 128 + row];
  const float l1 = dsmem_ld(theirs + (C * 128 + row) * 4);
  const float sk = p.sink != nullptr ? p.sink[h] : -INFINITY;
  const float m = fmaxf(fmaxf(l0, l1), sk);
  float w0 = 0.f, w1 = 0.f, den = 0.f;
  if (m > -INFINITY) {
    w0 = __expf(l0 - m);
    w1 = __expf(l1 - m);
    den = w0 + w1 + __expf(sk - m);
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  w0 *= inv;
  w1 *= inv;
  uint4* dst = reinterpret_cast<uint4*>(p.out + orow * C);
#pragma unroll 4
  for (int c8 = 0; c8 < C / 8; ++c8) {
    float4 a[2], b[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int v4 = 2 * c8 + u;
      a[u] = w0 > 0.f ? *reinterpret_cast<const float4*>(own + (v4 * 128 + row) * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
      b[u] = w1 > 0.f ? dsmem_ld4(theirs + (v4 * 128 + row) * 16) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    uint4 o;
    o.x = pack_bf16(w0 * a[0].x + w1 * b[0].x, w0 * a[0].y + w1 * b[0].y);
    o.y = pack_bf16(w0 * a[0].z + w1 * b[0].z, w0 * a[0].w + w1 * b[0].w);
    o.z = pack_bf16(w0 * a[1].x + w1 * b[1].x, w0 * a[1].y + w1 * b[1].y);
    o.w = pack_bf16(w0 * a[1].z + w1 * b[1].z, w0 * a[1].w + w1 * b[1].w);
    dst[c8] = o;
  }
  p.lse[orow] = den > 0.f ? m + __logf(den) : -INFINITY;
}

template <int C, int QB, int NS, int POLY8, bool CLUSTER>
__global__ void __launch_bounds__(PrefillLayout<C, QB, NS>::THREADS, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                   const PrefillParams p) {
  using L = PrefillLayout<C, QB, NS>;
  constexpr int BM = L::BM, BN = L::BN, SUB = L::SUB, IR = L::IR;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sKV = smem + L::OFF_KV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + QB;
  uint64_t* kv_full = q_empty + QB;
  uint64_t* kv_empty = kv_full + NS;
  uint64_t* s_full = kv_empty + NS;  // [warpgroup]: one phase per key tile
  uint64_t* p_half = s_full + 2;     // [warpgroup]: the first 64 keys' P of the tile is in TMEM
  uint64_t* p_ready = p_half + 2;    // [warpgroup]: all of the tile's P is in TMEM
  uint64_t* o_final = p_ready + 2;   // [warpgroup]: one phase per item, after its last P V
  uint64_t* o_free = o_final + 2;    // [warpgroup]: the epilogue has read O
  uint64_t* item_full = o_free + 2;
  uint64_t* item_empty = item_full + IR;
  uint64_t* q_stored = item_empty + IR;  // [QB]: both warpgroups are done with the buffer as output staging
  int2* s_items = reinterpret_cast<int2*>(smem + L::OFF_ITEM);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < QB; ++s) {
      mbar_init(q_full + s, 1);
      mbar_init(q_empty + s, 1);
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(kv_full + s, 1);
      mbar_init(kv_empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(s_full + s, 1);
      mbar_init(p_half + s, 128);
      mbar_init(p_ready + s, 128);
      mbar_init(o_final + s, 1);
      mbar_init(o_free + s, 128);
    }
    for (int s = 0; s < IR; ++s) {
      mbar_init(item_full + s, 1);
      mbar_init(item_empty + s, L::ITEM_READERS);
    }
    for (int s = 0; s < QB; ++s) mbar_init(q_stored + s, 2);
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
  const uint32_t tmem = *s_tmem;  // S_A at column 0, S_B at 128, O_A at 256, O_B at 256 + C

  // Each role ends with its own __syncthreads (the CTA's last barrier), so
  // no code runs under two different register limits.
  if (warp >= 8) {
  setmaxnreg_dec<L::REGS_CONTROL>();
  if (warp == L::LOAD_WARP) {
    // ------------------------------------------------------------ TMA loader
    bool ok = true;
    int idx = 0, g = 0, n = 0;  // items seen, key tiles issued, items with key tiles
    int pend_g = -1, pend_n0 = 0, pend_b = 0;  // (lane 0) the V tile not yet issued
    // ring entry u: K or V of a key tile starting at row n0 of batch row b
    auto load = [&](int u, bool v, int n0, int b) {
      const int slot = u % NS;
      if (u >= NS && !(ok = mbar_wait(kv_empty + slot, ((u / NS) & 1) ^ 1, p.status))) return;
      mbar_expect_tx(kv_full + slot, L::KV_BYTES);
      for (int s = 0; s < SUB; ++s)
        tma_load_3d(sKV + slot * L::KV_BYTES + s * BN * 128, v ? &tm_v : &tm_k, kv_full + slot, s * 64, n0, b);
    };
    for (int k = blockIdx.x; ok && k < p.items; k += gridDim.x, ++idx) {
      const PrefillItem it = prefill_item(p, k);  // the whole warp
      if (lane == 0) {
        const int slot = idx % IR;
        if (idx >= IR) ok = mbar_wait(item_empty + slot, ((idx / IR) & 1) ^ 1, p.status);
        if (ok) {
          s_items[slot] = make_int2(it.tile0, it.ntiles);
          mbar_arrive(item_full + slot);
        }
        for (int j = 0; ok && j < it.ntiles; ++j) {
          const int n0 = (it.tile0 + j) * BN;
          load(prefill_k_entry(g + j), false, n0, it.b);
          if (ok && pend_g >= 0) load(prefill_v_entry(pend_g), true, pend_n0, pend_b);
          pend_g = g + j;
          pend_n0 = n0;
          pend_b = it.b;
          if (ok && j == 0) {  // the Q pair, once the previous item's last V is on its way
            const int kn = k + static_cast<int>(gridDim.x);
            if (kn < p.items) {  // the next item's Q pair into L2 now, so that its load is an L2 hit
              const PrefillItem nx = prefill_place(p, kn);
              for (int w = 0; w < 2; ++w)
                for (int s = 0; s < SUB; ++s)
                  tma_prefetch_l2_2d(&tm_q, s * 64, (nx.b * p.T + nx.t0 + w * p.TQ) * p.H);
            }
            const int qb = n % QB;
            // the buffer's last item: its products have read Q, and its
            // output (staged there) has left
            if (n >= QB)
              ok = mbar_wait(q_empty + qb, ((n / QB) & 1) ^ 1, p.status) &&
                   mbar_wait(q_stored + qb, ((n / QB) & 1) ^ 1, p.status);
            if (ok) {
              mbar_expect_tx(q_full + qb, L::Q_BYTES);
              for (int w = 0; w < 2; ++w) {
                const int qrow0 = (it.b * p.T + it.t0 + w * p.TQ) * p.H;
                for (int s = 0; s < SUB; ++s)
                  tma_load_2d(sQ + qb * L::Q_BYTES + w * L::QT_BYTES + s * BM * 128, &tm_q, q_full + qb, s * 64,
                              qrow0);
              }
            }
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (it.ntiles > 0) {
        g += it.ntiles;
        ++n;
      }
    }
    if (lane == 0 && ok && pend_g >= 0) load(prefill_v_entry(pend_g), true, pend_n0, pend_b);
    // the consumers wait for every copy issued here before the CTA leaves
    // (or time out together with this thread), so nothing lands after exit
    if constexpr (CLUSTER) {  // the softmax warpgroups' two cluster barriers
      cluster_sync();
      cluster_sync();
    }
    tc_fence_before();
    __syncthreads();
  } else if (warp == L::MMA_WARP) {
    // ------------------------------------------------------ tcgen05 issuer
    const uint32_t q_addr = smem_u32(sQ), kv_addr = smem_u32(sKV);
    bool ok = true;
    int idx = 0, g = 0, n = 0;
    for (int k = blockIdx.x; ok && k < p.items; k += gridDim.x, ++idx) {
      const int slot = idx % IR;
      ok = mbar_wait(item_full + slot, (idx / IR) & 1, p.status);
      const int2 info = s_items[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(item_empty + slot);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const int nt = info.y;
      if (nt == 0) continue;
      // the whole warp runs the issue loop; one elected lane issues
      auto wait = [&](uint64_t* bar, int parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.status));
      };
      const int qb = n % QB;
      const uint32_t qa = q_addr + qb * L::Q_BYTES;
      // the ring entries a round reads are waited for at the end of the round
      // before, while the tensor pipe still has that round's products queued
      auto wait_kv = [&](int u) { return wait(kv_full + u % NS, (u / NS) & 1); };
      ok = wait(q_full + qb, (n / QB) & 1) && wait_kv(prefill_k_entry(g));
      if (ok) {
        tc_fence_after();
        prefill_issue_s<C, NS, L::QT_BYTES, L::KV_BYTES>(tmem, qa, kv_addr, 0, g, s_full);
        prefill_issue_s<C, NS, L::QT_BYTES, L::KV_BYTES>(tmem, qa, kv_addr, 1, g, s_full);
        mma_commit_warp(kv_empty + prefill_k_entry(g) % NS);
        if (nt == 1) mma_commit_warp(q_empty + qb);  // the item's last reader of Q
        ok = wait_kv(prefill_v_entry(g)) && (nt == 1 || wait_kv(prefill_k_entry(g + 1)));
      }
      for (int j = 1; ok && j <= nt; ++j) {
        const int gp = g + j - 1, gs = g + j;
        // warpgroup A: P V of tile j - 1 (by halves of P), then S of tile j
        if (!(ok = wait(p_half, gp & 1))) break;
        if (j == 1 && n >= 1 && !(ok = wait(o_free, (n - 1) & 1))) break;
        tc_fence_after();
        prefill_issue_pv<C, NS, L::KV_BYTES, 0>(tmem, kv_addr, 0, gp, j == 1);
        if (!(ok = wait(p_ready, gp & 1))) break;
        tc_fence_after();
        prefill_issue_pv<C, NS, L::KV_BYTES, 1>(tmem, kv_addr, 0, gp, j == 1);
        if (j == nt) mma_commit_warp(o_final);
        if (j < nt) prefill_issue_s<C, NS, L::QT_BYTES, L::KV_BYTES>(tmem, qa, kv_addr, 0, gs, s_full);
        // warpgroup B
        if (!(ok = wait(p_half + 1, gp & 1))) break;
        if (j == 1 && n >= 1 && !(ok = wait(o_free + 1, (n - 1) & 1))) break;
        tc_fence_after();
        prefill_issue_pv<C, NS, L::KV_BYTES, 0>(tmem, kv_addr, 1, gp, j == 1);
        if (!(ok = wait(p_ready + 1, gp & 1))) break;
        tc_fence_after();
        prefill_issue_pv<C, NS, L::KV_BYTES, 1>(tmem, kv_addr, 1, gp, j == 1);
        mma_commit_warp(kv_empty + prefill_v_entry(gp) % NS);
        if (j == nt) mma_commit_warp(o_final + 1);
        if (j < nt) {
          prefill_issue_s<C, NS, L::QT_BYTES, L::KV_BYTES>(tmem, qa, kv_addr, 1, gs, s_full);
          mma_commit_warp(kv_empty + prefill_k_entry(gs) % NS);
          if (j == nt - 1) mma_commit_warp(q_empty + qb);
          ok = wait_kv(prefill_v_entry(gs)) && (j + 1 == nt || wait_kv(prefill_k_entry(gs + 1)));
        }
      }
      g += nt;
      ++n;
    }
    if constexpr (CLUSTER) {
      cluster_sync();
      cluster_sync();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  } else {
    if constexpr (CLUSTER) {
      cluster_sync();
      cluster_sync();
    }
    tc_fence_before();
    __syncthreads();
  }
  } else {
    setmaxnreg_inc<L::REGS_SOFTMAX>();
    // ------------------- softmax: warpgroup w owns query tile w of the pair
    const int quad = warp & 3, w = warp >> 2;
    const int row = quad * 32 + lane;
    const int tq = row / p.H, h = row - tq * p.H;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t sAddr = lane_addr + w * 128, oAddr = lane_addr + 256 + w * C;
    const float sl2 = p.scale_log2;
    const int64_t rows_all = static_cast<int64_t>(p.B) * p.T * p.H;
    bool ok = true;
    int idx = 0, g = 0, n = 0;
    for (int k = blockIdx.x; ok && k < p.items; k += gridDim.x, ++idx) {
      const int slot = idx % IR;
      ok = mbar_wait(item_full + slot, (idx / IR) & 1, p.status);
      const int2 info = s_items[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(item_empty + slot);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const PrefillItem it = prefill_place(p, k);
      const int tile0 = info.x, nt = info.y;
      const int t = it.t0 + w * p.TQ + tq;
      const bool valid = tq < p.TQ && t < p.T;
      const int64_t orow = (static_cast<int64_t>(it.b) * p.T + t) * p.H + h;
      if (nt == 0) {  // an empty split: nothing to read
        if (valid) {
          if constexpr (CLUSTER) {  // its stash: no rows (the K/V ring is idle: nothing was loaded)
            reinterpret_cast<float*>(sKV + w * L::STASH_BYTES)[C * 128 + row] = -INFINITY;
          } else if (p.splits > 1) {
            p.part_lse[static_cast<int64_t>(it.split) * rows_all + orow] = -INFINITY;
          } else {
            for (int c = 0; c < C; ++c) p.out[orow * C + c] = __float2bfloat16_rn(0.f);
            p.lse[orow] = p.sink != nullptr ? p.sink[h] : -INFINITY;
          }
        }
        continue;
      }
      int lo = 1, hi = 0;  // an invalid row sees nothing
      if (valid) prefill_query_rows(p, it.b, t, lo, hi);
      int64_t tbase = int64_t(1) << 62;  // no tree: a base no row reaches
      uint64_t tbits = ~0ull;
      if (valid && p.tree_bits) {
        tbase = p.tree_base[it.b];
        tbits = p.tree_bits[static_cast<int64_t>(it.b) * p.T + t];
      }
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nt; ++j) {
        const int gs = g + j;
        ok = __all_sync(0xffffffffu, mbar_wait(s_full + w, gs & 1, p.status));
        if (!ok) break;
        tc_fence_after();
        uint32_t r[128];
        tmem_ld128(sAddr, r);
        const int n0 = (tile0 + j) * BN;  // the tile's first key
        const int a = lo - n0, b = hi - n0;  // the row sees tile columns a..b
        const bool in_tree = static_cast<int64_t>(n0) + BN > tbase && static_cast<int64_t>(n0) < tbase + 64;
        if (a > 0 || b < BN - 1 || in_tree) {
          const int tb = in_tree ? static_cast<int>(tbase - n0) : 0;  // the tree's first tile column
          prefill_mask_half(*reinterpret_cast<uint32_t(*)[64]>(r), 0, a, b, in_tree, tb, tbits);
          prefill_mask_half(*reinterpret_cast<uint32_t(*)[64]>(r + 64), 64, a, b, in_tree, tb, tbits);
        }
        const float tmax = max128(r) * sl2;
        const bool need = tmax > m_used + 8.f;
        const float alpha = need ? fast_exp2(m_used - tmax) : 1.f;
        if (need) {
          l *= alpha;
          m_used = tmax;
        }
        // S_w(gs) complete means P_w V of the tile before is too: O_w may be
        // rescaled (before p_half lets the next product accumulate into it)
        if (__any_sync(0xffffffffu, need) && j > 0) prefill_rescale_o<C>(oAddr, alpha);
        const float msub = m_used == -INFINITY ? 0.f : m_used;
        // P in two halves of 64 keys: the issuer starts on the first half's
        // product while the second half is computed
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t pk[32];
          float hmax;
          l += prefill_half_weights<POLY8>(*reinterpret_cast<const uint32_t(*)[64]>(r + 64 * hf), sl2, msub, pk, hmax);
          tmem_st32(sAddr + 32 * hf, pk);
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive((hf == 0 ? p_half : p_ready) + w);
        }
      }
      if (!ok) break;
      // o_final completes once per item, after the item's last P V product
      ok = __all_sync(0xffffffffu, mbar_wait(o_final + w, n & 1, p.status));
      if (!ok) break;
      tc_fence_after();
      uint32_t o[C];
      if constexpr (C == 128) {
        tmem_ld128(oAddr, o);
      } else {
        tmem_ld64(oAddr, o);
      }
      tc_fence_before();
      mbar_arrive(o_free + w);  // O_w may be overwritten by the next item
      const float msub = m_used == -INFINITY ? 0.f : m_used;
      float denom = l;
      if (p.splits == 1 && p.sink != nullptr && valid) denom += fast_exp2(fmaf(p.sink[h], LOG2E, -msub));
      const float inv = denom > 0.f ? 1.f / denom : 0.f;
      // A full query tile's output goes through its own Q buffer (free once
      // o_final says every product of the item is done): bf16 rows in the
      // 128-byte-swizzled layout of the TMA box, then one TMA store per 64
      // columns; the buffer is handed back to the loader (q_stored) once the
      // store has read it. Other tiles store their rows directly.
      if constexpr (CLUSTER) {  // the stash goes into the K/V ring: the other tile's products must be done too
        ok = __all_sync(0xffffffffu, mbar_wait(o_final + (w ^ 1), n & 1, p.status));
        if (!ok) break;
      }
      const bool stage = p.tma_out && p.splits == 1 && p.TQ * p.H == BM && it.t0 + (w + 1) * p.TQ <= p.T;
      uint8_t* tile = sQ + (n % QB) * L::Q_BYTES + w * L::QT_BYTES;
      if (stage) {
#pragma unroll
        for (int v4 = 0; v4 < C / 8; ++v4) {
          uint4 u;
          u.x = pack_bf16(__uint_as_float(o[v4 * 8 + 0]) * inv, __uint_as_float(o[v4 * 8 + 1]) * inv);
          u.y = pack_bf16(__uint_as_float(o[v4 * 8 + 2]) * inv, __uint_as_float(o[v4 * 8 + 3]) * inv);
          u.z = pack_bf16(__uint_as_float(o[v4 * 8 + 4]) * inv, __uint_as_float(o[v4 * 8 + 5]) * inv);
          u.w = pack_bf16(__uint_as_float(o[v4 * 8 + 6]) * inv, __uint_as_float(o[v4 * 8 + 7]) * inv);
          *reinterpret_cast<uint4*>(tile + (v4 >> 3) * (BM * 128) + sw128_offset(row, v4 & 7)) = u;
        }
        p.lse[orow] = denom > 0.f ? (msub + log2f(denom)) * LN2 : -INFINITY;
        fence_proxy_async();
        named_barrier(1 + w, 128);
        if (quad == 0 && lane == 0) {
          const int row0 = static_cast<int>((static_cast<int64_t>(it.b) * p.T + it.t0 + w * p.TQ) * p.H);
          for (int s = 0; s < SUB; ++s) tma_store_2d(&tm_o, tile + s * (BM * 128), s * 64, row0);
          bulk_commit();
          bulk_wait_read();
          mbar_arrive(q_stored + n % QB);
        }
      } else if (valid) {
        if (p.splits == 1) {
          uint4* dst = reinterpret_cast<uint4*>(p.out + orow * C);
#pragma unroll
          for (int v4 = 0; v4 < C / 8; ++v4) {
            uint4 u;
            u.x = pack_bf16(__uint_as_float(o[v4 * 8 + 0]) * inv, __uint_as_float(o[v4 * 8 + 1]) * inv);
            u.y = pack_bf16(__uint_as_float(o[v4 * 8 + 2]) * inv, __uint_as_float(o[v4 * 8 + 3]) * inv);
            u.z = pack_bf16(__uint_as_float(o[v4 * 8 + 4]) * inv, __uint_as_float(o[v4 * 8 + 5]) * inv);
            u.w = pack_bf16(__uint_as_float(o[v4 * 8 + 6]) * inv, __uint_as_float(o[v4 * 8 + 7]) * inv);
            dst[v4] = u;
          }
          p.lse[orow] = denom > 0.f ? (msub + log2f(denom)) * LN2 : -INFINITY;
        } else if constexpr (CLUSTER) {  // this split's normalised partial of the row, for the pair's combine
          float* st = reinterpret_cast<float*>(sKV + w * L::STASH_BYTES);
#pragma unroll
          for (int v4 = 0; v4 < C / 4; ++v4)
            *reinterpret_cast<float4*>(st + (v4 * 128 + row) * 4) =
                make_float4(__uint_as_float(o[v4 * 4]) * inv, __uint_as_float(o[v4 * 4 + 1]) * inv,
                            __uint_as_float(o[v4 * 4 + 2]) * inv, __uint_as_float(o[v4 * 4 + 3]) * inv);
          st[C * 128 + row] = l > 0.f ? (msub + log2f(l)) * LN2 : -INFINITY;
        } else {
          const int64_t prow = static_cast<int64_t>(it.split) * rows_all + orow;
          float4* dst = reinterpret_cast<float4*>(p.part_o + prow * C);
#pragma unroll
          for (int v4 = 0; v4 < C / 4; ++v4)
            dst[v4] = make_float4(__uint_as_float(o[v4 * 4]) * inv, __uint_as_float(o[v4 * 4 + 1]) * inv,
                                  __uint_as_float(o[v4 * 4 + 2]) * inv, __uint_as_float(o[v4 * 4 + 3]) * inv);
          p.part_lse[prow] = l > 0.f ? (msub + log2f(l)) * LN2 : -INFINITY;
        }
      }
      if (!stage && quad == 0 && lane == 0) mbar_arrive(q_stored + n % QB);
      g += nt;
      ++n;
    }
    if (quad == 0 && lane == 0) bulk_wait_all();  // this warpgroup's output stores have landed
    if constexpr (CLUSTER) {
      // every role of both CTAs comes here (after a time-out too), so the
      // cluster barriers always complete: the pair's stashes are written,
      // tile w's rows are combined by the CTA of rank w, and the partner's
      // stash is read before either CTA leaves
      cluster_sync();
      if (w == static_cast<int>(cluster_rank())) prefill_cluster_combine<C, L::STASH_BYTES>(p, sKV, w, row);
      cluster_sync();
    }
    tc_fence_before();
    __syncthreads();
  }
}

}  // namespace wpt
