// Backward pass of MQA attention over contiguous key ranges (one key-value
// head), tcgen05 + TMEM + TMA on sm_100a.
//
// Gradients of WPT's exact attention (packages/wpt-model/src/wpt_model/
// pytorch_kernels.py:123-139) and of its window/sink form (the window rows
// of :189-210; attention.py:85-107), from the forward pass's output and
// log-sum-exp. For a query row (token t, head h) with weights p_n over the
// rows lo_t..hi_t it reads:
//     delta = sum_c dO[c] O[c]
//     dS_n  = p_n (dO . v_n - delta)              (dz_n = scale * dS_n)
//     dQ    = scale * sum_n dS_n k_n
//     dK_n  = scale * sum_rows dS_n q,   dV_n = sum_rows p_n dO
//     d_sink[h] = -sum_rows exp(sink_h - lse) delta
// p_n = exp(z_n - lse) is recomputed from the saved log-sum-exp, as the
// reference does; P and dS enter the tensor-core products as bf16.
//
// Three kernels (query tiles are the forward's: TQ = 128 / H tokens x H
// heads = 128 rows of one batch row):
//   bwd_prep_kernel  one CTA per query tile: delta and lse * log2(e) per
//                    row (laid out per tile for one bulk copy), each token's
//                    rows lo..hi, the tile's key range, and per-tile partial
//                    sums of the sink's gradient (bwd_sink_kernel adds them
//                    in a fixed order, so d_sink is deterministic).
//   bwd_kv_kernel    one CTA per (key tile, batch row): the keys are the
//                    MMA's M, so dK and dV accumulate in TMEM over every query
//                    tile that sees the key tile, and each CTA writes its key
//                    tile's gradients once (no atomics):
//                      S^T  = K Q^T      A=K (smem),    B=Q (smem)
//                      dP^T = V dO^T     A=V (smem),    B=dO (smem)
//                      dV  += P^T dO     A=P^T (TMEM),  B=dO (smem, MN-major)
//                      dK  += dS^T Q     A=dS^T (TMEM), B=Q (smem, MN-major)
//   bwd_q_kernel     one CTA per query tile: the rows are the MMA's M and the
//                    key tiles stream through a ring:
//                      S = Q K^T, dP = dO V^T, dQ += dS K (A=dS in TMEM,
//                      B=K MN-major)
// Seven tile products per (query tile, key tile) pair against the five of a
// single kernel that adds dQ by atomics: the dQ pass recomputes S and dP
// instead, and every gradient is written exactly once.
//
// Warps (both main kernels): warps 0-7 compute P and dS, warp w reading TMEM
// lane quadrant w % 4 and column half w / 4 (64 of the tile's 128 columns),
// one thread per lane; warp 8 loads by TMA (one lane), warp 9 issues the
// products (one elected lane). TMEM: S at column 0, dP at 128, the
// accumulators at 256 (and 384). P and dS are written as bf16 pairs over
// the first 64 columns of S and dP; a named barrier between the loads of a
// tile's S and dP and those writes keeps one half's writes from landing on
// the other half's unread columns.
//
// Every mbarrier wait is bounded (common.cuh); a wait that runs out sets
// the status word and every role stops, the compute warps together (their
// barrier ANDs the flag).
#pragma once

#include <climits>

#include "common.cuh"
#include "prefill.cuh"
#include "stream.cuh"

namespace wpt {

constexpr int BWD_THREADS = 320;
constexpr int BWD_LOAD_WARP = 8, BWD_MMA_WARP = 9, BWD_COMPUTE = 256;

struct BwdParams {
  const int64_t* positions;    // (B, T) each query's own row
  const int64_t* floor_rows;   // (B, T) or null: the lowest row each query reads
  const __nv_bfloat16* out;    // (B, T, H, C) the forward pass's output
  const __nv_bfloat16* d_out;  // (B, T, H, C)
  const float* lse;            // (B, T, H) natural log, sink included
  const float* sink;           // (H,) or null
  float* ld;                   // (B, qtiles, 2, 128) scratch: lse * log2(e), then delta, per tile row
  int2* ranges;                // (B, qtiles) scratch: lowest and highest key row the tile reads
  int2* bounds;                // (B, T) scratch: each token's rows lo..hi
  float* sink_part;            // (B * qtiles, H) scratch: per-tile sums of exp(sink - lse) * delta
  void* dq;                    // (B, T, H, C)
  void* dk;                    // (B, N, C)
  void* dv;                    // (B, N, C)
  float* d_sink;               // (H,) or null
  unsigned* status;
  int B, T, H, N, window, TQ, qtiles, ktiles;
  int f32_grads;  // 1: dq, dk, dv in fp32 (a gathered-rows pass adds to them after), 0: bf16
  float scale, scale_log2;
  // the query-tile kernel's wait limit, and (a failure-detection test hook,
  // -1 when off) a key tile whose copy its loader does not issue, so that
  // the waits for it run out while nothing is in flight
  unsigned long long wait_ns;
  int skip_key_tile;
  // the key-tile kernel's work split: each key tile's query tiles in
  // kv_parts equal ranges of tile indices, one CTA each; with more than one
  // part each CTA writes fp32 partial dK, dV (kv_part, (parts, B, N, 256):
  // dK then dV) and bwd_kv_reduce_kernel adds them in part order
  int kv_parts;
  float* kv_part;
};

// Rows lo..hi query t of batch row b reads (hi < lo: none): hi = min(p, N - 1),
// lo = max(0, p - window + 1 when window > 0, floor).
__device__ __forceinline__ int2 bwd_token_rows(const BwdParams& p, int b, int t) {
  const int64_t pos = p.positions[static_cast<int64_t>(b) * p.T + t];
  const int64_t top = pos < static_cast<int64_t>(p.N) - 1 ? pos : static_cast<int64_t>(p.N) - 1;
  int64_t low = 0;
  if (p.window > 0 && pos - p.window + 1 > low) low = pos - p.window + 1;
  if (p.floor_rows) {
    const int64_t f = p.floor_rows[static_cast<int64_t>(b) * p.T + t];
    if (f > low) low = f;
  }
  return make_int2(low > INT_MAX ? INT_MAX : static_cast<int>(low), top < -1 ? -1 : static_cast<int>(top));
}

__device__ __forceinline__ float bf16_dot8(uint4 a, uint4 b) {
  const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* y = reinterpret_cast<const __nv_bfloat162*>(&b);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 u = __bfloat1622float2(x[i]), v = __bfloat1622float2(y[i]);
    s = fmaf(u.x, v.x, s);
    s = fmaf(u.y, v.y, s);
  }
  return s;
}

// One CTA of 128 threads per (query tile j, batch row b); thread r owns tile
// row r (token j * TQ + r / H, head r % H). C = 128.
__global__ void __launch_bounds__(128) bwd_prep_kernel(const BwdParams p) {
  const int j = blockIdx.x, b = blockIdx.y, r = threadIdx.x;
  const int lane = r & 31, warp = r >> 5;
  const int tq = r / p.H, h = r - tq * p.H;
  const int t = j * p.TQ + tq;
  const bool valid = tq < p.TQ && t < p.T;
  __shared__ float s_sink[128];
  __shared__ float s_delta[128];
  __shared__ int s_lo[4], s_hi[4];
  if (r < p.H) s_sink[r] = 0.f;
  // delta = rowsum(dO * O) of the warp's 32 rows: per step each half-warp
  // reads one row of O and dO (16 lanes x 16 bytes, coalesced) and sums its
  // dot product over the half
  {
    const int half = lane >> 4, ch = lane & 15;
#pragma unroll 4
    for (int k = 0; k < 16; ++k) {
      const int rr = warp * 32 + 2 * k + half;
      const int tq2 = rr / p.H, t2 = j * p.TQ + tq2;
      float d = 0.f;
      if (tq2 < p.TQ && t2 < p.T) {
        const int64_t row2 = (static_cast<int64_t>(b) * p.T + t2) * p.H + (rr - tq2 * p.H);
        d = bf16_dot8(reinterpret_cast<const uint4*>(p.out + row2 * 128)[ch],
                      reinterpret_cast<const uint4*>(p.d_out + row2 * 128)[ch]);
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      if (ch == 0) s_delta[rr] = d;
    }
  }
  __syncthreads();
  float lse2 = 0.f, delta = 0.f;
  int lo = INT_MAX, hi = -1;
  if (valid) {
    const int64_t row = (static_cast<int64_t>(b) * p.T + t) * p.H + h;
    delta = s_delta[r];
    const float l = p.lse[row];
    lse2 = l * LOG2E;
    // a row that reads nothing has lse = sink (or -inf without one) and out = 0
    if (p.sink != nullptr && l != -INFINITY) atomicAdd(&s_sink[h], __expf(p.sink[h] - l) * delta);
    const int2 bt = bwd_token_rows(p, b, t);
    if (h == 0) p.bounds[static_cast<int64_t>(b) * p.T + t] = bt;
    if (bt.y >= bt.x) {
      lo = bt.x;
      hi = bt.y;
    }
  }
  float* ld = p.ld + (static_cast<int64_t>(b) * p.qtiles + j) * 256;
  ld[r] = lse2;
  ld[128 + r] = delta;
  lo = __reduce_min_sync(0xffffffffu, lo);
  hi = __reduce_max_sync(0xffffffffu, hi);
  if (lane == 0) {
    s_lo[warp] = lo;
    s_hi[warp] = hi;
  }
  __syncthreads();
  if (r == 0) {
    int a = s_lo[0], z = s_hi[0];
    for (int w = 1; w < 4; ++w) {
      a = min(a, s_lo[w]);
      z = max(z, s_hi[w]);
    }
    p.ranges[static_cast<int64_t>(b) * p.qtiles + j] = make_int2(a, z);
  }
  if (p.sink != nullptr && r < p.H)
    p.sink_part[(static_cast<int64_t>(b) * p.qtiles + j) * p.H + r] = s_sink[r];
}

// d_sink[h] = -(sum over the tiles' partial sums), one CTA per head, a fixed
// order of additions.
__global__ void __launch_bounds__(256) bwd_sink_kernel(const float* __restrict__ part, int64_t tiles, int H,
                                                       float* __restrict__ d_sink) {
  const int h = blockIdx.x;
  __shared__ float s_red[8];
  float acc = 0.f;
  for (int64_t i = threadIdx.x; i < tiles; i += 256) acc += part[i * H + h];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.f;
    for (int w = 0; w < 8; ++w) total += s_red[w];
    d_sink[h] = -total;
  }
}

// Whether query tile j of batch row b reads any key of the tile at n0.
__device__ __forceinline__ bool bwd_tile_sees(const BwdParams& p, int b, int j, int n0) {
  const int2 r = p.ranges[static_cast<int64_t>(b) * p.qtiles + j];
  return r.y >= r.x && r.x <= n0 + 127 && r.y >= n0;
}

// 64 fp32 values of one thread (a TMEM row's half) to global memory at dst,
// as bf16 (f32 == 0) or fp32, times mul.
__device__ __forceinline__ void bwd_store64(void* dst, const uint32_t (&v)[64], float mul, int f32) {
  if (f32) {
    float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int i = 0; i < 16; ++i)
      d[i] = make_float4(__uint_as_float(v[4 * i]) * mul, __uint_as_float(v[4 * i + 1]) * mul,
                         __uint_as_float(v[4 * i + 2]) * mul, __uint_as_float(v[4 * i + 3]) * mul);
  } else {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint4 u;
      u.x = pack_bf16(__uint_as_float(v[8 * i + 0]) * mul, __uint_as_float(v[8 * i + 1]) * mul);
      u.y = pack_bf16(__uint_as_float(v[8 * i + 2]) * mul, __uint_as_float(v[8 * i + 3]) * mul);
      u.z = pack_bf16(__uint_as_float(v[8 * i + 4]) * mul, __uint_as_float(v[8 * i + 5]) * mul);
      u.w = pack_bf16(__uint_as_float(v[8 * i + 6]) * mul, __uint_as_float(v[8 * i + 7]) * mul);
      d[i] = u;
    }
  }
}

// The first query tile at or after j that reads a key of the tile at n0
// (qtiles when none). Warp-collective: the lanes test 32 tiles with one load
// each and a ballot keeps the answer (base, mask) for the next calls, so a
// key tile that most query tiles skip costs a load per 32 tiles, not one
// per tile.
struct BwdTileScan {
  int base = -64;
  uint32_t mask = 0;
  // the first query tile in [j, end) that reads the key tile at n0, or end
  __device__ __forceinline__ int next(const BwdParams& p, int b, int n0, int j, int end) {
    const int lane = threadIdx.x & 31;
    while (j < end) {
      if (j >= base + 32) {
        base = j & ~31;
        const int jj = base + lane;
        mask = __ballot_sync(0xffffffffu, jj < end && bwd_tile_sees(p, b, jj, n0));
      }
      const uint32_t m = mask & (0xffffffffu << (j - base));
      if (m) return min(end, base + __ffs(m) - 1);
      j = base + 32;
    }
    return end;
  }
};

// Work of one key-tile CTA: key tile n0 / 128 of batch row b, its query
// tiles [jbeg, jend), part `part` of kv_parts. Order: key tile 0 (under a
// causal mask the most read) of every part and batch row first, then tile 1, ...
struct BwdKvUnit {
  int b, n0, part, jbeg, jend;
};
__device__ __forceinline__ BwdKvUnit bwd_kv_place(const BwdParams& p) {
  const int idx = static_cast<int>(blockIdx.x);
  BwdKvUnit w;
  const int per_tile = p.kv_parts * p.B;
  w.n0 = (idx / per_tile) * 128;
  const int rem = idx - (idx / per_tile) * per_tile;
  w.part = rem / p.B;
  w.b = rem - w.part * p.B;
  w.jbeg = static_cast<int>(static_cast<int64_t>(w.part) * p.qtiles / p.kv_parts);
  w.jend = static_cast<int>(static_cast<int64_t>(w.part + 1) * p.qtiles / p.kv_parts);
  return w;
}

// Where a key-tile CTA's dK and dV rows go: the gradients themselves (one
// part) or the unit's fp32 partials.
__device__ __forceinline__ void bwd_kv_store(const BwdParams& p, const BwdKvUnit& w, int n, int g,
                                             const uint32_t (&gv)[64], const uint32_t (&gk)[64]) {
  if (p.kv_parts > 1) {
    float* row = p.kv_part + ((static_cast<int64_t>(w.part) * p.B + w.b) * p.N + n) * 256 + 64 * g;
    bwd_store64(row, gk, p.scale, 1);
    bwd_store64(row + 128, gv, 1.f, 1);
  } else {
    const int64_t off = (static_cast<int64_t>(w.b) * p.N + n) * 128 + 64 * g;
    const int es = p.f32_grads ? 4 : 2;
    bwd_store64(static_cast<uint8_t*>(p.dv) + off * es, gv, 1.f, p.f32_grads);
    bwd_store64(static_cast<uint8_t*>(p.dk) + off * es, gk, p.scale, p.f32_grads);
  }
}

// dK, dV = the sum of the key-tile CTAs' fp32 partials, in part order
// (deterministic), to bf16 or fp32. One thread per 4 values.
__global__ void __launch_bounds__(256) bwd_kv_reduce_kernel(const float* __restrict__ part, int parts, int64_t rows,
                                                            void* dk, void* dv, int f32) {
  const int64_t n4 = rows * 64;  // 256 floats a row, 4 a thread
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 acc = reinterpret_cast<const float4*>(part)[i];
    for (int q = 1; q < parts; ++q) {
      const float4 x = reinterpret_cast<const float4*>(part + q * rows * 256)[i];
      acc.x += x.x;
      acc.y += x.y;
      acc.z += x.z;
      acc.w += x.w;
    }
    const int64_t row = i / 64, c4 = i - row * 64;  // dK columns 0..127 (c4 < 32), then dV
    const int64_t o = row * 128 + (c4 & 31) * 4;
    void* dst = c4 < 32 ? dk : dv;
    if (f32) {
      *reinterpret_cast<float4*>(static_cast<float*>(dst) + o) = acc;
    } else {
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(dst) + o) =
          make_uint2(pack_bf16(acc.x, acc.y), pack_bf16(acc.z, acc.w));
    }
  }
}

struct BwdKvLayout {
  static constexpr int TILE = 128 * 128 * 2;     // a 128 x 128 bf16 tile, two 64-column chunks
  static constexpr int CHUNK = 128 * 128;        // bytes between the chunks
  static constexpr int NSQ = 2;                  // query-tile stages
  static constexpr int STAGE = 2 * TILE + 1024;  // Q, dO, then lse * log2(e) and delta (2 x 128 fp32)
  static constexpr int OFF_K = 0, OFF_V = TILE, OFF_ST = 2 * TILE;
  static constexpr int OFF_BAR = OFF_ST + NSQ * STAGE;
  // kv_full, st_full[NSQ], st_empty[NSQ], s_full[2], p_ready[2], acc_done
  static constexpr int NBAR = 6 + 2 * NSQ;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16 + 1024;
};

__global__ void __launch_bounds__(BWD_THREADS, 1)
    bwd_kv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                  const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                  const BwdParams p) {
  using L = BwdKvLayout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* st_full = kv_full + 1;
  uint64_t* st_empty = st_full + L::NSQ;
  uint64_t* s_full = st_empty + L::NSQ;  // [half]: S^T and dP^T of the tile's half are in TMEM
  uint64_t* p_ready = s_full + 2;        // [half]: its P^T and dS^T are
  uint64_t* acc_done = p_ready + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const BwdKvUnit w = bwd_kv_place(p);
  const int b = w.b, n0 = w.n0, jbeg = w.jbeg, jend = w.jend;
  {
    // a unit no query tile of its range reads: zero gradients, no TMEM,
    // no loads (every warp's scan gives the same answer)
    BwdTileScan pre;
    if (pre.next(p, b, n0, jbeg, jend) >= jend) {
      const uint32_t zero[64] = {};
      for (int r = threadIdx.x; r < 2 * 128; r += blockDim.x) {
        const int n = n0 + (r >> 1);
        if (n < p.N) bwd_kv_store(p, w, n, r & 1, zero, zero);
      }
      return;
    }
  }

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < L::NSQ; ++s) {
      mbar_init(st_full + s, 1);
      mbar_init(st_empty + s, 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(s_full + g, 1);
      mbar_init(p_ready + g, BWD_COMPUTE / 2);
    }
    mbar_init(acc_done, 1);
    fence_mbar_init();
  }
  if (warp == BWD_MMA_WARP) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  if (warp == BWD_LOAD_WARP && lane == 0) {
    tma_prefetch(&tm_q);
    tma_prefetch(&tm_do);
    tma_prefetch(&tm_k);
    tma_prefetch(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;  // S^T at 0, dP^T at 128, dV at 256, dK at 384

  if (warp == BWD_LOAD_WARP) {
    // ------------------------------------------------------------ TMA loader
    // the whole warp scans the query tiles; lane 0 issues the copies
    bool ok = true;
    if (lane == 0) {
      mbar_expect_tx(kv_full, 2 * L::TILE);
      for (int s = 0; s < 2; ++s) {
        tma_load_3d(smem + L::OFF_K + s * L::CHUNK, &tm_k, kv_full, s * 64, n0, b);
        tma_load_3d(smem + L::OFF_V + s * L::CHUNK, &tm_v, kv_full, s * 64, n0, b);
      }
    }
    BwdTileScan scan;
    int u = 0;
    for (int j = scan.next(p, b, n0, jbeg, jend); ok && j < jend; j = scan.next(p, b, n0, j + 1, jend), ++u) {
      const int st = u % L::NSQ;
      if (lane == 0) {
        if (u >= L::NSQ) ok = mbar_wait(st_empty + st, ((u / L::NSQ) & 1) ^ 1, p.status);
        if (ok) {
          uint8_t* stage = smem + L::OFF_ST + st * L::STAGE;
          mbar_expect_tx(st_full + st, 2 * L::TILE + 1024);
          const int row0 = (b * p.T + j * p.TQ) * p.H;
          for (int s = 0; s < 2; ++s) {
            tma_load_2d(stage + s * L::CHUNK, &tm_q, st_full + st, s * 64, row0);
            tma_load_2d(stage + L::TILE + s * L::CHUNK, &tm_do, st_full + st, s * 64, row0);
          }
          bulk_load(stage + 2 * L::TILE, p.ld + (static_cast<int64_t>(b) * p.qtiles + j) * 256, 1024,
                    st_full + st);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    tc_fence_before();
    __syncthreads();
  } else if (warp == BWD_MMA_WARP) {
    // ------------------------------------------------------ tcgen05 issuer
    // A query tile's rows come in two halves of 64 (g = 0, 1), one per
    // compute warpgroup. Order: S_0 dP_0 S_1 dP_1 of tile u, then per tile
    // dV/dK of half 0, S_0 dP_0 of tile u + 1, dV/dK of half 1, S_1 dP_1 of
    // tile u + 1: each warpgroup's P and dS are computed while the tensor
    // pipe runs the other half's products. tcgen05 products run in issue
    // order, so S_g of the next tile overwrites P_g only after dV has read it.
    auto wait = [&](uint64_t* bar, int parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.status));
    };
    const uint32_t base = smem_u32(smem);
    const uint64_t dk = sdesc_sw128(base + L::OFF_K, 16, 1024), dv = sdesc_sw128(base + L::OFF_V, 16, 1024);
    auto issue_s = [&](int uu, int g) {  // S^T_g = K Q_g^T and dP^T_g = V dO_g^T (N = 64 query rows)
      const uint32_t stage = base + L::OFF_ST + (uu % L::NSQ) * L::STAGE + g * 64 * 128;
      prefill_s_steps<7>(tmem + 64 * g, dk, sdesc_sw128(stage, 16, 1024), idesc_bf16(128, 64, 0, 0));
      prefill_s_steps<7>(tmem + 128 + 64 * g, dv, sdesc_sw128(stage + L::TILE, 16, 1024), idesc_bf16(128, 64, 0, 0));
      mma_commit_warp(s_full + g);
    };
    auto issue_acc = [&](int uu, int g, uint32_t acc0) {  // dV += P_g^T dO_g, dK += dS_g^T Q_g (K = 64 rows)
      const uint32_t stage = base + L::OFF_ST + (uu % L::NSQ) * L::STAGE + g * 64 * 128;
      prefill_pv_steps<3, 0>(tmem + 256, tmem + 64 * g, sdesc_sw128(stage + L::TILE, L::CHUNK, 1024),
                             idesc_bf16(128, 128, 0, 1), acc0);
      prefill_pv_steps<3, 0>(tmem + 384, tmem + 128 + 64 * g, sdesc_sw128(stage, L::CHUNK, 1024),
                             idesc_bf16(128, 128, 0, 1), acc0);
    };
    bool ok = wait(kv_full, 0);
    BwdTileScan scan;
    int j = scan.next(p, b, n0, jbeg, jend);
    if (ok && j < jend && (ok = wait(st_full, 0))) {
      tc_fence_after();
      issue_s(0, 0);
      issue_s(0, 1);
    }
    for (int u = 0; ok && j < jend; ++u) {
      const int jn = scan.next(p, b, n0, j + 1, jend);
      if (!(ok = wait(p_ready, u & 1))) break;
      tc_fence_after();
      issue_acc(u, 0, u > 0 ? 1u : 0u);
      if (jn < jend) {
        if (!(ok = wait(st_full + (u + 1) % L::NSQ, ((u + 1) / L::NSQ) & 1))) break;
        tc_fence_after();
        issue_s(u + 1, 0);
      }
      if (!(ok = wait(p_ready + 1, u & 1))) break;
      tc_fence_after();
      issue_acc(u, 1, 1u);
      mma_commit_warp(st_empty + u % L::NSQ);
      if (jn < jend) issue_s(u + 1, 1);
      j = jn;
    }
    mma_commit_warp(acc_done);  // once every product above has completed
    wait(acc_done, 0);  // so that no product or commit is in flight at the dealloc (bounded)
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  } else {
    // ----------------------- P and dS: warpgroup g owns the tiles' half g
    const int quad = warp & 3, g = warp >> 2;
    const int row = quad * 32 + lane, n = n0 + row;  // this thread's key
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint64_t sl2 = f2_pack(p.scale_log2, p.scale_log2);
    bool ok = true;
    BwdTileScan scan;
    int u = 0;
    for (int j = scan.next(p, b, n0, jbeg, jend); ok && j < jend; j = scan.next(p, b, n0, j + 1, jend), ++u) {
      const int st = u % L::NSQ;
      const float* lds = reinterpret_cast<const float*>(smem + L::OFF_ST + st * L::STAGE + 2 * L::TILE);
      // the columns (query rows 64 g + c) that see key n, by token (global
      // loads issued before the waits below, so their latency hides)
      uint64_t vis = 0;
      const int c0 = 64 * g;
      for (int tq = c0 / p.H; tq < p.TQ && tq * p.H < c0 + 64; ++tq) {
        const int t = j * p.TQ + tq;
        if (t >= p.T) break;
        const int2 bt = p.bounds[static_cast<int64_t>(b) * p.T + t];
        if (n >= bt.x && n <= bt.y) {
          const int a = max(tq * p.H, c0) - c0, z = min(tq * p.H + p.H, c0 + 64) - c0;  // columns a .. z - 1
          const uint64_t hi_mask = z >= 64 ? ~0ull : ((1ull << z) - 1ull);
          vis |= hi_mask & ~((1ull << a) - 1ull);
        }
      }
      // the stage's copies (its lse and delta are read here) and the half's
      // S^T and dP^T; the stage is not refilled before this thread's
      // p_ready arrival, so the parity names this use of it
      ok = __all_sync(0xffffffffu, mbar_wait(st_full + st, (u / L::NSQ) & 1, p.status) &&
                                       mbar_wait(s_full + g, u & 1, p.status));
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {  // 32 columns at a time; a thread's writes only land on columns it has read
        uint32_t s[32], d[32];
        tmem_ld32x2(lane_addr + 64 * g + 32 * ch, lane_addr + 128 + 64 * g + 32 * ch, s, d);
        uint32_t pk[16], dsk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int c = c0 + 32 * ch + 2 * i;
          const uint64_t z = f2_fma(f2_pack(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])), sl2,
                                    f2_pack(-lds[c], -lds[c + 1]));
          float z0, z1, e0, e1;
          f2_unpack(z, z0, z1);
          if ((i & 3) == 3) {  // a quarter of the exponentials on the FMA pipe, the rest on the exp unit
            exp2_poly_pair(z0, z1, e0, e1);
          } else {
            e0 = fast_exp2(z0);
            e1 = fast_exp2(z1);
          }
          const int bit = 32 * ch + 2 * i;
          e0 = (vis >> bit) & 1ull ? e0 : 0.f;
          e1 = (vis >> (bit + 1)) & 1ull ? e1 : 0.f;
          const uint64_t gd = f2_add(f2_pack(__uint_as_float(d[2 * i]), __uint_as_float(d[2 * i + 1])),
                                     f2_pack(-lds[128 + c], -lds[128 + c + 1]));
          float g0, g1;
          f2_unpack(gd, g0, g1);
          pk[i] = pack_bf16(e0, e1);
          dsk[i] = pack_bf16(e0 * g0, e1 * g1);
        }
        tmem_st16(lane_addr + 64 * g + 16 * ch, pk);         // P^T_g over S^T_g's first 32 columns
        tmem_st16(lane_addr + 128 + 64 * g + 16 * ch, dsk);  // dS^T_g over dP^T_g's
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_ready + g);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(acc_done, 0, p.status));
    tc_fence_after();
    uint32_t gv[64], gk[64];
    if (ok && u > 0) {
      tmem_ld64(lane_addr + 256 + 64 * g, gv);
      tmem_ld64(lane_addr + 384 + 64 * g, gk);
    } else {
#pragma unroll
      for (int i = 0; i < 64; ++i) gv[i] = gk[i] = 0u;
    }
    if (ok && n < p.N) bwd_kv_store(p, w, n, g, gv, gk);
    tc_fence_before();
    __syncthreads();
  }
}

struct BwdQLayout {
  static constexpr int TILE = 128 * 128 * 2, CHUNK = 128 * 128;
  static constexpr int NS = 2;  // key-tile stages (K and V)
  static constexpr int OFF_Q = 0, OFF_DO = TILE, OFF_LD = 2 * TILE;
  static constexpr int OFF_KV = 2 * TILE + 1024;
  static constexpr int STAGE = 2 * TILE;
  static constexpr int OFF_BAR = OFF_KV + NS * STAGE;
  // q_full, kv_full[NS], kv_empty[NS], s_full[2], ds_ready[2], acc_done
  static constexpr int NBAR = 6 + 2 * NS;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16 + 1024;
};

__global__ void __launch_bounds__(BWD_THREADS, 1)
    bwd_q_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                 const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                 const BwdParams p) {
  using L = BwdQLayout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;
  uint64_t* kv_empty = kv_full + L::NS;
  uint64_t* s_full = kv_empty + L::NS;  // [half]: S and dP of the key tile's half are in TMEM
  uint64_t* ds_ready = s_full + 2;      // [half]: its dS is
  uint64_t* acc_done = ds_ready + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // later query tiles read more keys: the last tile of every batch row first
  const int b = static_cast<int>(blockIdx.x) % p.B, j = p.qtiles - 1 - static_cast<int>(blockIdx.x) / p.B;
  const int2 rg = p.ranges[static_cast<int64_t>(b) * p.qtiles + j];
  const int kt0 = rg.y >= rg.x ? rg.x / 128 : 0;
  const int nt = rg.y >= rg.x ? rg.y / 128 - kt0 + 1 : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < L::NS; ++s) {
      mbar_init(kv_full + s, 1);
      mbar_init(kv_empty + s, 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(s_full + g, 1);
      mbar_init(ds_ready + g, BWD_COMPUTE / 2);
    }
    mbar_init(acc_done, 1);
    fence_mbar_init();
  }
  if (warp == BWD_MMA_WARP) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  if (warp == BWD_LOAD_WARP && lane == 0) {
    tma_prefetch(&tm_q);
    tma_prefetch(&tm_do);
    tma_prefetch(&tm_k);
    tma_prefetch(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;  // S at 0, dP at 128, dQ at 256

  if (warp == BWD_LOAD_WARP) {
    if (lane == 0) {
      bool ok = true;
      const int row0 = (b * p.T + j * p.TQ) * p.H;
      mbar_expect_tx(q_full, 2 * L::TILE + 1024);
      for (int s = 0; s < 2; ++s) {
        tma_load_2d(smem + L::OFF_Q + s * L::CHUNK, &tm_q, q_full, s * 64, row0);
        tma_load_2d(smem + L::OFF_DO + s * L::CHUNK, &tm_do, q_full, s * 64, row0);
      }
      bulk_load(smem + L::OFF_LD, p.ld + (static_cast<int64_t>(b) * p.qtiles + j) * 256, 1024, q_full);
      int last[L::NS];  // the last use of each stage whose copies were issued (-1: none)
      for (int st = 0; st < L::NS; ++st) last[st] = -1;
      for (int i = 0; ok && i < nt; ++i) {
        const int st = i % L::NS;
        if (i >= L::NS && !(ok = mbar_wait_ns(kv_empty + st, ((i / L::NS) & 1) ^ 1, p.status, p.wait_ns))) break;
        if (i == p.skip_key_tile) continue;  // test hook: this tile's copy is never issued
        uint8_t* stage = smem + L::OFF_KV + st * L::STAGE;
        mbar_expect_tx(kv_full + st, 2 * L::TILE);
        for (int s = 0; s < 2; ++s) {
          tma_load_3d(stage + s * L::CHUNK, &tm_k, kv_full + st, s * 64, (kt0 + i) * 128, b);
          tma_load_3d(stage + L::TILE + s * L::CHUNK, &tm_v, kv_full + st, s * 64, (kt0 + i) * 128, b);
        }
        last[st] = i;
      }
      if (!ok) {
        // a wait ran out: the copies issued here land before the CTA leaves
        // (each stage's last issued use, and the query tile's), bounded too
        mbar_wait_ns(q_full, 0, p.status, p.wait_ns);
        for (int st = 0; st < L::NS; ++st)
          if (last[st] >= 0) mbar_wait_ns(kv_full + st, (last[st] / L::NS) & 1, p.status, p.wait_ns);
      }
    }
    tc_fence_before();
    __syncthreads();
  } else if (warp == BWD_MMA_WARP) {
    // the key tile's two halves of 64 keys (g = 0, 1), one per compute
    // warpgroup, in the key-tile kernel's order: dQ += dS_0 K_0, the next
    // tile's S_0 dP_0, dQ += dS_1 K_1, the next tile's S_1 dP_1
    auto wait = [&](uint64_t* bar, int parity) {
      return __all_sync(0xffffffffu, mbar_wait_ns(bar, parity, p.status, p.wait_ns));
    };
    const uint32_t base = smem_u32(smem);
    const uint64_t dq = sdesc_sw128(base + L::OFF_Q, 16, 1024), ddo = sdesc_sw128(base + L::OFF_DO, 16, 1024);
    auto issue_s = [&](int i, int g) {  // S_g = Q K_g^T, dP_g = dO V_g^T (N = 64 keys)
      const uint32_t stage = base + L::OFF_KV + (i % L::NS) * L::STAGE + g * 64 * 128;
      prefill_s_steps<7>(tmem + 64 * g, dq, sdesc_sw128(stage, 16, 1024), idesc_bf16(128, 64, 0, 0));
      prefill_s_steps<7>(tmem + 128 + 64 * g, ddo, sdesc_sw128(stage + L::TILE, 16, 1024), idesc_bf16(128, 64, 0, 0));
      mma_commit_warp(s_full + g);
    };
    auto issue_dq = [&](int i, int g, uint32_t acc0) {  // dQ += dS_g K_g (K = 64 keys, K_g MN-major)
      const uint32_t stage = base + L::OFF_KV + (i % L::NS) * L::STAGE + g * 64 * 128;
      prefill_pv_steps<3, 0>(tmem + 256, tmem + 128 + 64 * g, sdesc_sw128(stage, L::CHUNK, 1024),
                             idesc_bf16(128, 128, 0, 1), acc0);
    };
    bool ok = wait(q_full, 0);
    if (ok && nt > 0 && (ok = wait(kv_full, 0))) {
      tc_fence_after();
      issue_s(0, 0);
      issue_s(0, 1);
    }
    for (int i = 0; ok && i < nt; ++i) {
      if (!(ok = wait(ds_ready, i & 1))) break;
      tc_fence_after();
      issue_dq(i, 0, i > 0 ? 1u : 0u);
      if (i + 1 < nt) {
        if (!(ok = wait(kv_full + (i + 1) % L::NS, ((i + 1) / L::NS) & 1))) break;
        tc_fence_after();
        issue_s(i + 1, 0);
      }
      if (!(ok = wait(ds_ready + 1, i & 1))) break;
      tc_fence_after();
      issue_dq(i, 1, 1u);
      mma_commit_warp(kv_empty + i % L::NS);
      if (i + 1 < nt) issue_s(i + 1, 1);
    }
    mma_commit_warp(acc_done);
    wait(acc_done, 0);  // so that no product or commit is in flight at the dealloc (bounded)
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  } else {
    // ------------------------- dS: warpgroup g owns the key tiles' half g
    const int quad = warp & 3, g = warp >> 2;
    const int row = quad * 32 + lane;  // this thread's query row
    const int tq = row / p.H, h = row - tq * p.H;
    const int t = j * p.TQ + tq;
    const bool valid = tq < p.TQ && t < p.T;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float sl2 = p.scale_log2;
    int2 bt = make_int2(1, 0);
    if (valid) bt = p.bounds[static_cast<int64_t>(b) * p.T + t];
    bool ok = __all_sync(0xffffffffu, mbar_wait_ns(q_full, 0, p.status, p.wait_ns));
    const float* lds = reinterpret_cast<const float*>(smem + L::OFF_LD);
    const float lse2 = lds[row], delta = lds[128 + row];
    const uint64_t sl2p = f2_pack(sl2, sl2), nl = f2_pack(-lse2, -lse2), nd = f2_pack(-delta, -delta);
    for (int i = 0; ok && i < nt; ++i) {
      ok = __all_sync(0xffffffffu, mbar_wait_ns(s_full + g, i & 1, p.status, p.wait_ns));
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {  // 32 keys at a time; a thread's writes only land on columns it has read
        const int nb = (kt0 + i) * 128 + 64 * g + 32 * ch;  // these columns' first key
        const int a = bt.x - nb, z = bt.y - nb;            // visible columns a .. z
        uint32_t s[32], d[32];
        tmem_ld32x2(lane_addr + 64 * g + 32 * ch, lane_addr + 128 + 64 * g + 32 * ch, s, d);
        uint32_t dsk[16];
#pragma unroll
        for (int k2 = 0; k2 < 16; ++k2) {
          const int c = 2 * k2;
          const uint64_t zz = f2_fma(f2_pack(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), sl2p, nl);
          float z0, z1, e0, e1;
          f2_unpack(zz, z0, z1);
          if ((k2 & 3) == 3) {  // a quarter of the exponentials on the FMA pipe
            exp2_poly_pair(z0, z1, e0, e1);
          } else {
            e0 = fast_exp2(z0);
            e1 = fast_exp2(z1);
          }
          e0 = c >= a && c <= z ? e0 : 0.f;
          e1 = c + 1 >= a && c + 1 <= z ? e1 : 0.f;
          const uint64_t gd = f2_add(f2_pack(__uint_as_float(d[c]), __uint_as_float(d[c + 1])), nd);
          float g0, g1;
          f2_unpack(gd, g0, g1);
          dsk[k2] = pack_bf16(e0 * g0, e1 * g1);
        }
        tmem_st16(lane_addr + 128 + 64 * g + 16 * ch, dsk);  // dS_g over dP_g's first 32 columns
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(ds_ready + g);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait_ns(acc_done, 0, p.status, p.wait_ns));
    tc_fence_after();
    uint32_t gq[64];
    if (ok && nt > 0) {
      tmem_ld64(lane_addr + 256 + 64 * g, gq);
    } else {
#pragma unroll
      for (int i = 0; i < 64; ++i) gq[i] = 0u;
    }
    if (ok && valid) {
      const int64_t off = ((static_cast<int64_t>(b) * p.T + t) * p.H + h) * 128 + 64 * g;
      bwd_store64(static_cast<uint8_t*>(p.dq) + off * (p.f32_grads ? 4 : 2), gq, p.scale, p.f32_grads);
    }
    tc_fence_before();
    __syncthreads();
  }
}

// ------------------------------------------------- gathered rows (sparse)
//
// The chosen-row share of sparse attention's gradients
// (pytorch_kernels.py:189-210 over idx; the window rows are the range
// kernels' share, added to the same fp32 gradients). One CTA per query
// (b, t), its K chosen rows in tiles of 128 gathered rows, the rows as the
// MMA's M and the query's heads (padded to NCOL = 16, 32 or 64) as N:
//   S^T  = K_g Q^T        A=K_g (smem),          B=Q (smem)
//   dP^T = V_g dO^T       A=V_g (smem),          B=dO (smem)
//   dV_g = P^T dO         A=P^T (TMEM),          B=dO (smem, MN-major)
//   dK_g = dS^T Q         A=dS^T (TMEM),         B=Q (smem, MN-major)
//   dQ^T += K_g^T dS^T    A=K_g (smem, MN-major), B=dS^T (smem)
// dV_g and dK_g rows are added into the fp32 gradients of the rows they
// belong to (vector atomics: different queries choose the same rows); dQ^T
// accumulates in TMEM over the tiles and is added to the query's fp32 dq
// (which only this CTA touches) at the end.
// Warps 0-3 (one TMEM lane quadrant each, thread = gathered row, or channel
// at the end) compute P and dS; warp 4 allocates TMEM and issues; warps 5-6
// gather the rows by 16-byte cp.async into the swizzled tiles.

constexpr int GBWD_THREADS = 224, GBWD_LOADERS = 64;

struct GatherBwdParams {
  const __nv_bfloat16* q;      // (B, T, H, C)
  const __nv_bfloat16* d_out;  // (B, T, H, C)
  const __nv_bfloat16* k;      // table rows at k + b * ksb + n * ksn
  const __nv_bfloat16* v;
  int64_t ksb, ksn, vsb, vsn;
  const int64_t* idx;          // (B, T, K), -1 for none
  const float* ld;             // the prep kernel's per-tile lse * log2(e) and delta
  float* dq;                   // (B, T, H, C) fp32, added to
  float* dk;                   // (B, N, C) fp32, added to
  float* dv;                   // (B, N, C) fp32, added to
  unsigned* status;
  int B, T, H, N, K, TQ, qtiles;
  float scale, scale_log2;
};

template <int NCOL>
struct GatherBwdLayout {
  static constexpr int QT = NCOL * 128 * 2;     // Q or dO: NCOL rows x 128 columns, two chunks
  static constexpr int TILE = 128 * 128 * 2;   // a gathered K or V tile
  static constexpr int OFF_Q = 0, OFF_DO = QT, OFF_DS = 2 * QT;  // dS^T: NCOL rows x 128 gathered rows
  static constexpr int OFF_KV = ((3 * QT + 1023) / 1024) * 1024;
  static constexpr int STAGE = 2 * TILE;       // K_g then V_g
  static constexpr int NS = 2;
  static constexpr int OFF_ROWS = OFF_KV + NS * STAGE;  // int [NS][128]
  static constexpr int OFF_LD = OFF_ROWS + NS * 128 * 4;  // lse2[64], delta[64]
  static constexpr int OFF_BAR = OFF_LD + 128 * 4;
  // q_full, full[NS], kv_empty[NS], s_full, p_ready, acc_ready, acc_free
  static constexpr int NBAR = 5 + 2 * NS;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16 + 1024;
};

template <int NCOL>
__device__ __forceinline__ void gbwd_ld(uint32_t taddr, uint32_t (&r)[NCOL]) {
  if constexpr (NCOL == 16) {
    tmem_ld16(taddr, r);
  } else if constexpr (NCOL == 32) {
    tmem_ld32(taddr, r);
  } else {
    tmem_ld64(taddr, r);
  }
}

template <int NW>
__device__ __forceinline__ void gbwd_st(uint32_t taddr, const uint32_t (&r)[NW]) {
  if constexpr (NW == 8) {
    uint32_t x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = i < 8 ? r[i] : 0u;
    tmem_st16(taddr, x);  // the upper 8 columns are not read (K = 16 heads)
  } else if constexpr (NW == 16) {
    tmem_st16(taddr, r);
  } else {
    tmem_st32(taddr, r);
  }
}

template <int NCOL>
__global__ void __launch_bounds__(GBWD_THREADS, 1) bwd_gather_kernel(const GatherBwdParams p) {
  using L = GatherBwdLayout<NCOL>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  int* s_rows = reinterpret_cast<int*>(smem + L::OFF_ROWS);
  float* s_l2 = reinterpret_cast<float*>(smem + L::OFF_LD);
  float* s_dl = s_l2 + 64;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* full = q_full + 1;
  uint64_t* kv_empty = full + L::NS;
  uint64_t* s_full = kv_empty + L::NS;
  uint64_t* p_ready = s_full + 1;
  uint64_t* acc_ready = p_ready + 1;
  uint64_t* acc_free = acc_ready + 1;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bt = blockIdx.x;  // the query (b, t)
  const int b = static_cast<int>(bt / p.T), t = static_cast<int>(bt - static_cast<int64_t>(b) * p.T);
  const int ntiles = (p.K + 127) / 128;

  if (threadIdx.x == 0) {
    mbar_init(q_full, GBWD_LOADERS);
    for (int s = 0; s < L::NS; ++s) {
      mbar_init(full + s, GBWD_LOADERS);
      mbar_init(kv_empty + s, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_ready, 128);
    mbar_init(acc_ready, 1);
    mbar_init(acc_free, 128);
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;  // S^T 0, dP^T 64, dV_g 128, dK_g 256, dQ^T 384

  if (warp >= 5) {
    // --------------------------------------------------------- loaders
    const int lt = threadIdx.x - 160;
    const int64_t qrow = (static_cast<int64_t>(b) * p.T + t) * p.H;
    for (int it = lt; it < NCOL * 16; it += GBWD_LOADERS) {
      const int h = it >> 4, ch = it & 15;
      const bool ok = h < p.H;
      const int64_t off = (qrow + (ok ? h : 0)) * 128 + ch * 8;
      const uint32_t dst = (ch >> 3) * (NCOL * 128) + sw128_offset(h, ch & 7);
      cp_async_16(smem_u32(smem + L::OFF_Q + dst), p.q + off, ok);
      cp_async_16(smem_u32(smem + L::OFF_DO + dst), p.d_out + off, ok);
    }
    if (lt < 64) {
      const int j = t / p.TQ, r0 = (t - j * p.TQ) * p.H;
      const float* ld = p.ld + (static_cast<int64_t>(b) * p.qtiles + j) * 256;
      s_l2[lt] = lt < p.H ? ld[r0 + lt] : 0.f;
      s_dl[lt] = lt < p.H ? ld[128 + r0 + lt] : 0.f;
    }
    cp_async_commit();
    cp_async_wait<0>();
    fence_proxy_async();
    mbar_arrive(q_full);
    const int64_t* idx = p.idx + bt * p.K;
    const uint8_t* kb = reinterpret_cast<const uint8_t*>(p.k + static_cast<int64_t>(b) * p.ksb);
    const uint8_t* vb = reinterpret_cast<const uint8_t*>(p.v + static_cast<int64_t>(b) * p.vsb);
    bool ok = true;
    for (int i = 0; ok && i < ntiles; ++i) {
      const int st = i % L::NS;
      if (i >= L::NS) ok = mbar_wait(kv_empty + st, ((i / L::NS) & 1) ^ 1, p.status);
      ok = named_barrier_and(2, GBWD_LOADERS, ok);
      if (!ok) break;
      uint8_t* stage = smem + L::OFF_KV + st * L::STAGE;
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {  // this thread's two rows of the tile
        const int r = lt + 64 * hr;
        const int slot = i * 128 + r;
        int64_t row = slot < p.K ? idx[slot] : -1;
        if (row < 0 || row >= p.N) row = -1;
        s_rows[st * 128 + r] = static_cast<int>(row);
        const bool live = row >= 0;
        const uint8_t* ks = kb + (live ? row : 0) * p.ksn * 2;
        const uint8_t* vs = vb + (live ? row : 0) * p.vsn * 2;
#pragma unroll
        for (int ch = 0; ch < 16; ++ch) {
          const uint32_t dst = (ch >> 3) * (128 * 128) + sw128_offset(r, ch & 7);
          cp_async_16(smem_u32(stage + dst), ks + ch * 16, live);
          cp_async_16(smem_u32(stage + L::TILE + dst), vs + ch * 16, live);
        }
      }
      cp_async_commit();
      cp_async_wait<0>();
      fence_proxy_async();
      mbar_arrive(full + st);
    }
    tc_fence_before();
    __syncthreads();
  } else if (warp == 4) {
    // ------------------------------------------------------------ issuer
    auto wait = [&](uint64_t* bar, int parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.status));
    };
    const uint32_t base = smem_u32(smem);
    const uint64_t dq_k = sdesc_sw128(base + L::OFF_Q, 16, 1024), ddo_k = sdesc_sw128(base + L::OFF_DO, 16, 1024);
    const uint64_t dq_mn = sdesc_sw128(base + L::OFF_Q, NCOL * 128, 1024);
    const uint64_t ddo_mn = sdesc_sw128(base + L::OFF_DO, NCOL * 128, 1024);
    const uint64_t dds = sdesc_sw128(base + L::OFF_DS, 16, 1024);
    bool ok = wait(q_full, 0);
    for (int i = 0; ok && i < ntiles; ++i) {
      const int st = i % L::NS;
      const uint32_t stage = base + L::OFF_KV + st * L::STAGE;
      if (!(ok = wait(full + st, (i / L::NS) & 1))) break;
      tc_fence_after();
      stream_s_steps<NCOL, 7>(tmem, sdesc_sw128(stage, 16, 1024), dq_k, idesc_bf16(128, NCOL, 0, 0));
      stream_s_steps<NCOL, 7>(tmem + 64, sdesc_sw128(stage + L::TILE, 16, 1024), ddo_k, idesc_bf16(128, NCOL, 0, 0));
      mma_commit_warp(s_full);
      if (!(ok = wait(p_ready, i & 1))) break;
      if (i > 0 && !(ok = wait(acc_free, (i - 1) & 1))) break;
      tc_fence_after();
      prefill_pv_steps<NCOL / 16 - 1, 0>(tmem + 128, tmem, ddo_mn, idesc_bf16(128, 128, 0, 1), 0u);      // dV_g
      prefill_pv_steps<NCOL / 16 - 1, 0>(tmem + 256, tmem + 64, dq_mn, idesc_bf16(128, 128, 0, 1), 0u);  // dK_g
      stream_pv_steps<NCOL, 7>(tmem + 384, sdesc_sw128(stage, 128 * 128, 1024), dds, idesc_bf16(128, NCOL, 1, 0),
                               i > 0 ? 1u : 0u);  // dQ^T += K_g^T dS^T
      mma_commit_warp(acc_ready);
      mma_commit_warp(kv_empty + st);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  } else {
    // -------------------------------------------- P and dS (warps 0-3)
    const int r = warp * 32 + lane;  // this thread's gathered row in each tile
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const float sl2 = p.scale_log2;
    uint8_t* sds = smem + L::OFF_DS;
    bool ok = __all_sync(0xffffffffu, mbar_wait(q_full, 0, p.status));
    for (int i = 0; ok && i < ntiles; ++i) {
      const int st = i % L::NS;
      ok = __all_sync(0xffffffffu,
                      mbar_wait(full + st, (i / L::NS) & 1, p.status) && mbar_wait(s_full, i & 1, p.status));
      if (!ok) break;
      tc_fence_after();
      const int row = s_rows[st * 128 + r];
      uint32_t s[NCOL], d[NCOL];
      gbwd_ld<NCOL>(lane_addr, s);
      gbwd_ld<NCOL>(lane_addr + 64, d);
      uint32_t pk[NCOL / 2], dsk[NCOL / 2];
#pragma unroll
      for (int h2 = 0; h2 < NCOL / 2; ++h2) {
        float pp[2], gg[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int h = 2 * h2 + e;
          const bool live = row >= 0 && h < p.H;
          pp[e] = live ? fast_exp2(fmaf(__uint_as_float(s[h]), sl2, -s_l2[h])) : 0.f;
          gg[e] = pp[e] * (__uint_as_float(d[h]) - s_dl[h]);
        }
        pk[h2] = pack_bf16(pp[0], pp[1]);
        dsk[h2] = pack_bf16(gg[0], gg[1]);
        // dS^T as the dQ product's B operand: head rows, gathered rows along K
        const __nv_bfloat162 g2 = __floats2bfloat162_rn(gg[0], gg[1]);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int h = 2 * h2 + e;
          const uint32_t off = (r >> 6) * (NCOL * 128) + sw128_offset(h, (r & 63) >> 3) + (r & 7) * 2;
          *reinterpret_cast<__nv_bfloat16*>(sds + off) = e == 0 ? g2.x : g2.y;
        }
      }
      gbwd_st<NCOL / 2>(lane_addr, pk);        // P^T over S^T's columns
      gbwd_st<NCOL / 2>(lane_addr + 64, dsk);  // dS^T over dP^T's columns
      fence_proxy_async();
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_ready);
      ok = __all_sync(0xffffffffu, mbar_wait(acc_ready, i & 1, p.status));
      if (!ok) break;
      tc_fence_after();
      // this row's shares of dV and dK, added into the gradients of table row `row`
#pragma unroll
      for (int c32 = 0; c32 < 4; ++c32) {
        uint32_t gv[32], gk[32];
        tmem_ld32(lane_addr + 128 + c32 * 32, gv);
        tmem_ld32(lane_addr + 256 + c32 * 32, gk);
        if (row >= 0) {
          float* dvr = p.dv + (static_cast<int64_t>(b) * p.N + row) * 128 + c32 * 32;
          float* dkr = p.dk + (static_cast<int64_t>(b) * p.N + row) * 128 + c32 * 32;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            atomicAdd(reinterpret_cast<float4*>(dvr) + e,
                      make_float4(__uint_as_float(gv[4 * e]), __uint_as_float(gv[4 * e + 1]),
                                  __uint_as_float(gv[4 * e + 2]), __uint_as_float(gv[4 * e + 3])));
            atomicAdd(reinterpret_cast<float4*>(dkr) + e,
                      make_float4(__uint_as_float(gk[4 * e]) * p.scale, __uint_as_float(gk[4 * e + 1]) * p.scale,
                                  __uint_as_float(gk[4 * e + 2]) * p.scale, __uint_as_float(gk[4 * e + 3]) * p.scale));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(acc_free);
    }
    if (ok) {
      // dQ^T: lane c of the four warps is channel c, NCOL head columns
      tc_fence_after();
      uint32_t g[NCOL];
      gbwd_ld<NCOL>(lane_addr + 384, g);
      const int c = r;
      float* dq = p.dq + bt * p.H * 128 + c;
      for (int h = 0; h < p.H; ++h) dq[h * 128] += __uint_as_float(g[h]) * p.scale;
    }
    tc_fence_before();
    __syncthreads();
  }
}

// fp32 gradients to bf16 (the sparse path accumulates in fp32).
__global__ void __launch_bounds__(256) f32_to_bf16_kernel(const float4* __restrict__ x, int64_t n4,
                                                          uint2* __restrict__ y) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 v = x[i];
    y[i] = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
  }
}

}  // namespace wpt
