// Key-stream attention for few queries per batch row: decode, short
// extends, and sparse attention over gathered rows. tcgen05 + TMEM on
// sm_100a, with the keys as the MMA's M:
//
//   S^T  = K Q^T     M = 128 keys, N = NCOL columns (query x head), K = C
//   O^T += V^T P^T   M = C,        N = NCOL,                        K = 128 keys
//
// so a single decode query's 32 heads still fill 128-row tensor-core tiles
// (the keys), where the prefill kernel's rows would be three-quarters
// empty. Replaces the decode use of exact_attention
// (packages/wpt-model/src/wpt_model/pytorch_kernels.py:98-121 at T = 1;
// the Triton form runs it on a (1, B) grid, triton_kernels.py:216) and
// sparse_attention (pytorch_kernels.py:171-187,213-217; the Triton form's
// _sparse_forward_kernel, triton_kernels.py:681-716).
//
// Keys. A CTA streams "slots" of one batch row. Range mode: slot i is row
// lo + i of the union of its queries' ranges (each query masks its own
// lo..hi). Gather mode (sparse): one query per CTA; slot i < K is
// idx[b, t, i], then the query's window rows p - window + 1 .. p; -1, or a
// row outside the table, is masked (pytorch_kernels.py:149-153,182).
// Slots are split into chunks of chunk_tiles x 128 over gridDim.y; with
// more than one split every CTA writes a partial result for the merge
// kernel (merge.cuh), or, in cluster mode (at most 8 splits, the grid one
// wave), the splits of a query group form one thread-block cluster: each
// CTA pushes (remote shared-memory stores) its unnormalised output and its
// columns' maximum and sum to the CTA that owns each column (column c: CTA
// c % splits), and after a cluster barrier every CTA combines its columns
// from its own shared memory and writes the final output, so neither
// partials in HBM nor a second launch.
//
// Loads: range mode takes whole tiles by TMA. Gather mode: 2 loader warps
// copy each slot's 256-byte K and V rows with 16-byte cp.async (coalesced:
// 16 lanes per row) into 128-byte-swizzled tiles and publish a stage after
// cp.async.wait_group and a proxy fence; a tile of the query's window rows
// (one contiguous range) comes by TMA instead. Q's copy is in flight
// together with the first tiles' (range mode: the first STAGES tiles' TMA
// loads are issued before it; gather mode: tile 0's copies follow it in
// the next cp.async group). Warp 4 issues the MMAs.
// Warps 0-3 do the softmax: thread r owns slot r of a tile, holds its
// NCOL scores, and the per-column maximum and sum over the 128 slots come
// from a 31-shuffle transpose reduction per warp plus shared memory across
// the four warps. P^T is written to shared memory (bf16) as the second
// MMA's B operand. The running maximum is lazy (raised only by more than
// 8 in base 2), as in the prefill kernel.
#pragma once

#include <climits>

#include "common.cuh"

namespace wpt {

struct StreamParams {
  const __nv_bfloat16* q;  // (B, T, H, C) contiguous
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t ksb, ksn, vsb, vsn;  // table strides, elements
  const int64_t* positions;    // (B, T)
  const int64_t* floor_rows;   // (B, T) or null (range mode)
  const int64_t* idx;          // (B, T, K) or null: gather mode
  const float* sink;           // (H,) or null
  __nv_bfloat16* out;          // (B, T, H, C)
  float* lse;                  // (B, T, H)
  float* part_o;               // (splits, B*T*H, C)
  float* part_lse;             // (splits, B*T*H)
  unsigned* status;
  int B, T, H, N, K, window, TQ, groups_per_row, splits, chunk_tiles;
  int window_tma;              // gather mode: tiles of window rows come by TMA (the maps are valid)
  int cluster;                 // > 1: the splits of a group are one cluster and merge in shared memory
  float scale_log2;
};

template <int NCOL, int STAGES>
struct StreamLayout {
  static constexpr int C = 128, BN = 128;
  static constexpr int Q_BYTES = NCOL * C * 2;
  static constexpr int KV_BYTES = BN * C * 2;
  static constexpr int P_BYTES = NCOL * BN * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = ((Q_BYTES + 1023) / 1024) * 1024;
  static constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr int OFF_P = OFF_V + STAGES * KV_BYTES;
  static constexpr int OFF_ROW = OFF_P + 2 * P_BYTES;
  static constexpr int OFF_RED = OFF_ROW + STAGES * BN * 4;
  static constexpr int OFF_M = OFF_RED + 4 * 64 * 4;
  static constexpr int OFF_ALPHA = OFF_M + 64 * 4;
  static constexpr int OFF_L = OFF_ALPHA + 64 * 4;
  static constexpr int OFF_QLO = OFF_L + 64 * 4;
  static constexpr int OFF_QHI = OFF_QLO + 64 * 4;
  static constexpr int OFF_COLQ = OFF_QHI + 64 * 4;
  static constexpr int OFF_BAR = OFF_COLQ + 64 * 4;
  static constexpr int NBAR = 1 + 2 * STAGES + 6;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16 + 1024;
  static constexpr int TMEM_COLS = 3 * NCOL <= 32 ? 32 : 3 * NCOL <= 64 ? 64 : 3 * NCOL <= 128 ? 128 : 256;
};

constexpr int STREAM_THREADS = 224;  // warps 0-3 softmax, 4 MMA, 5-6 loaders
constexpr int STREAM_LOADERS = 64;

__device__ __forceinline__ void stream_query_rows(const StreamParams& p, int b, int t, int& lo, int& hi) {
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

// S^T (+)= K Q^T over head-width steps 0..KK: A = the K tile (K-major,
// 64-element chunks BN * 128 bytes apart), B = Q (K-major, NCOL rows).
template <int NCOL, int KK>
__device__ __forceinline__ void stream_s_steps(uint32_t d, uint64_t dk, uint64_t dq, uint32_t idesc) {
  if constexpr (KK > 0) stream_s_steps<NCOL, KK - 1>(d, dk, dq, idesc);
  constexpr uint32_t off_k = ((KK >> 2) * (128 * 128) + (KK & 3) * 32) >> 4;
  constexpr uint32_t off_q = ((KK >> 2) * (NCOL * 128) + (KK & 3) * 32) >> 4;
  mma_ss_off_warp<off_k, off_q>(d, dk, dq, idesc, KK > 0 ? 1u : 0u);
}
// O^T (+)= V^T P^T over key steps 0..KK: A = V^T (MN-major), B = P^T
// (K-major, NCOL rows); acc0 = 0 makes the first step overwrite O^T.
template <int NCOL, int KK>
__device__ __forceinline__ void stream_pv_steps(uint32_t d, uint64_t dv, uint64_t dp, uint32_t idesc, uint32_t acc0) {
  if constexpr (KK > 0) stream_pv_steps<NCOL, KK - 1>(d, dv, dp, idesc, acc0);
  constexpr uint32_t off_v = (KK * 16 * 128) >> 4;
  constexpr uint32_t off_p = ((KK >> 2) * (NCOL * 128) + (KK & 3) * 32) >> 4;
  mma_ss_off_warp<off_v, off_p>(d, dv, dp, idesc, KK > 0 ? 1u : acc0);
}

// Cluster mode's combine, run by every thread of every CTA of the cluster
// (one query group's splits) after each CTA has left, for its columns, the
// lazy maximum (s_m, base 2), the sum of exponentials (s_l; 0 when the
// split saw no visible key or a wait failed) and the unnormalised output
// (s_o, 128 floats a column) in its own shared memory. CTA k owns columns
// k, k + S, ...: after a cluster barrier its threads read every split's
// (m, l) of those columns once (distributed shared memory loads), turn them
// into weights w_i / L (w_i = 2^(m_i - M) over the splits with l_i > 0, L =
// sum_i w_i l_i plus the sink's exp(sink - M), M their largest m), then each
// 4-float chunk of an owned column's output takes all S splits' chunks in
// one round of loads. A second barrier keeps every CTA's memory in place
// until the others have read it.
__device__ __forceinline__ void stream_cluster_merge(const StreamParams& p, const float* s_m, const float* s_l,
                                                     const float* s_o, float* s_w, int64_t row0, int ncols) {
  constexpr int C = 128;
  cluster_sync();
  const int S = p.cluster;
  const int rank = static_cast<int>(cluster_rank());
  const int mine = ncols > rank ? (ncols - rank + S - 1) / S : 0;  // columns rank, rank + S, ...
  const uint32_t am = smem_u32(s_m), al = smem_u32(s_l), ao = smem_u32(s_o);
  // s_w[cl * 9 + i]: split i's weight over L for owned column cl; s_w[cl * 9 + 8]: the log-sum
  if (static_cast<int>(threadIdx.x) < mine) {
    const int cl = threadIdx.x, c = rank + cl * S;
    float mi[8], li[8];
    float M = -INFINITY;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      mi[i] = -INFINITY;
      li[i] = 0.f;
      if (i < S) {
        mi[i] = dsmem_ld(dsmem_map(am + c * 4, i));
        li[i] = dsmem_ld(dsmem_map(al + c * 4, i));
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (li[i] > 0.f) M = fmaxf(M, mi[i]);
    const float msub = M == -INFINITY ? 0.f : M;
    float w[8], L = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      w[i] = li[i] > 0.f ? fast_exp2(mi[i] - msub) : 0.f;
      L = fmaf(w[i], li[i], L);
    }
    if (p.sink != nullptr) L += fast_exp2(fmaf(p.sink[c % p.H], LOG2E, -msub));
    const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s_w[cl * 9 + i] = w[i] * inv;
    s_w[cl * 9 + 8] = L > 0.f ? (msub + log2f(L)) * LN2 : -INFINITY;
  }
  __syncthreads();
  for (int item = threadIdx.x; item < mine * (C / 4); item += blockDim.x) {
    const int cl = item / (C / 4), quad = item % (C / 4), c = rank + cl * S;
    float4 o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < S && s_w[cl * 9 + i] != 0.f) o[i] = dsmem_ld4(dsmem_map(ao + (c * C + quad * 4) * 4, i));
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float w = i < S ? s_w[cl * 9 + i] : 0.f;
      if (w != 0.f) {
        acc.x = fmaf(w, o[i].x, acc.x);
        acc.y = fmaf(w, o[i].y, acc.y);
        acc.z = fmaf(w, o[i].z, acc.z);
        acc.w = fmaf(w, o[i].w, acc.w);
      }
    }
    uint2 packed;
    packed.x = pack_bf16(acc.x, acc.y);
    packed.y = pack_bf16(acc.z, acc.w);
    *reinterpret_cast<uint2*>(p.out + (row0 + c) * C + quad * 4) = packed;
    if (quad == 0) p.lse[row0 + c] = s_w[cl * 9 + 8];
  }
  cluster_sync();  // no CTA leaves while another still reads its shared memory
}

template <int NCOL, int STAGES, bool GATHER>
__global__ void __launch_bounds__(STREAM_THREADS, 1)
    stream_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                  const StreamParams p) {
  using L = StreamLayout<NCOL, STAGES>;
  constexpr int C = L::C, BN = L::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  uint8_t* sP = smem + L::OFF_P;
  int* s_row = reinterpret_cast<int*>(smem + L::OFF_ROW);
  float* s_red = reinterpret_cast<float*>(smem + L::OFF_RED);
  float* s_m = reinterpret_cast<float*>(smem + L::OFF_M);
  float* s_alpha = reinterpret_cast<float*>(smem + L::OFF_ALPHA);
  float* s_l = reinterpret_cast<float*>(smem + L::OFF_L);
  int* s_qlo = reinterpret_cast<int*>(smem + L::OFF_QLO);
  int* s_qhi = reinterpret_cast<int*>(smem + L::OFF_QHI);
  int* s_colq = reinterpret_cast<int*>(smem + L::OFF_COLQ);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* full = bars + 1;
  uint64_t* kv_empty = full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;
  uint64_t* p_ready = s_full + 2;
  uint64_t* o_done = p_ready + 2;
  uint64_t* o_final = o_done + 1;  // one phase: the last P V product has completed
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  int* s_range = reinterpret_cast<int*>(smem + L::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int group = blockIdx.x, split = blockIdx.y;
  const int b = group / p.groups_per_row;
  const int t0 = (group - b * p.groups_per_row) * p.TQ;
  const int TQg = min(p.TQ, p.T - t0);  // queries of this group
  constexpr bool gather = GATHER;
  const int64_t rows_total = static_cast<int64_t>(p.B) * p.T * p.H;

  // Set-up, one barrier: warp 0 reads the group's query positions (their
  // rows, and in range mode the union of their ranges) while warp 1 clears
  // the column state, warp 2 the unused query slots, warp 3 initialises the
  // mbarriers and warp 4 allocates TMEM.
  const int lane = threadIdx.x & 31;
  if (warp == 0) {
    // launched as a programmatic dependent of the kernel before it on the
    // stream: everything above runs while that kernel finishes, and nothing
    // in global memory is read or written before it has
    griddep_wait();
    int rlo = INT_MAX, rhi = -1;
    for (int tq = lane; tq < TQg; tq += 32) {
      int lo, hi;
      stream_query_rows(p, b, t0 + tq, lo, hi);
      s_qlo[tq] = lo;
      s_qhi[tq] = hi;
      if (hi >= lo) {
        rlo = min(rlo, lo);
        rhi = max(rhi, hi);
      }
    }
    rlo = __reduce_min_sync(0xffffffffu, rlo);
    rhi = __reduce_max_sync(0xffffffffu, rhi);
    if (lane == 0) {
      s_range[0] = rlo;
      s_range[1] = rhi;
    }
  } else if (warp == 1 || warp == 2) {
    for (int i = lane; i < 64; i += 32) {
      if (warp == 1) {
        s_m[i] = -INFINITY;
        const int tq = i / p.H;  // column -> its query in the group, -1 for padding
        s_colq[i] = (i < NCOL && tq < TQg) ? tq : -1;
      } else if (i >= TQg) {
        s_qlo[i] = 0;
        s_qhi[i] = -1;
      }
    }
  } else if (warp == 3 && lane == 0) {
    mbar_init(q_full, STREAM_LOADERS);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, GATHER ? STREAM_LOADERS : 1);
      mbar_init(kv_empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(s_full + s, 1);
      mbar_init(p_ready + s, 128);
    }
    mbar_init(o_done, 1);
    mbar_init(o_final, 1);
    fence_mbar_init();
  } else if (warp == 4) {
    tmem_alloc(s_tmem, L::TMEM_COLS);
    tmem_relinquish();
  }
  griddep_wait();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // this CTA's slots: [slot0, slot_end) of `total`
  int64_t total;
  int range_lo = 0;
  if (gather) {
    total = static_cast<int64_t>(p.K) + (p.window > 0 ? p.window : 0);
  } else {
    range_lo = s_range[0];
    total = s_range[1] >= s_range[0] ? static_cast<int64_t>(s_range[1]) - s_range[0] + 1 : 0;
  }
  const int64_t tiles_total = (total + BN - 1) / BN;
  // range mode: chunk_tiles consecutive tiles per split; gather mode: tiles
  // split, split + splits, ... (the window's contiguous tiles, loaded by TMA,
  // and the gathered ones spread evenly over the splits)
  const int64_t tile0 = static_cast<int64_t>(split) * p.chunk_tiles;
  const int64_t left = tiles_total - tile0;
  const int ntiles =
      GATHER ? static_cast<int>(split < tiles_total ? (tiles_total - split + gridDim.y - 1) / gridDim.y : 0)
             : static_cast<int>(left <= 0 ? 0 : (left < p.chunk_tiles ? left : p.chunk_tiles));
  // Gather mode takes its tiles alternately from the gathered slots (16-byte
  // copies, bounded by the requests an SM's L1 keeps in flight) and the
  // window's (TMA), so that both kinds of load are in flight together.
  const int64_t gathered_tiles = (static_cast<int64_t>(p.K) + BN - 1) / BN;  // tiles with a slot below K
  const int kg = GATHER ? static_cast<int>(gathered_tiles > split ? (gathered_tiles - split + gridDim.y - 1) / gridDim.y
                                                                  : 0)
                        : 0;
  const int kg_mine = kg < ntiles ? kg : ntiles;
  const int pairs = kg_mine < ntiles - kg_mine ? kg_mine : ntiles - kg_mine;
  auto tile_of = [&](int j) -> int64_t {
    if constexpr (!GATHER) {
      return tile0 + j;
    } else {
      int k;
      if (j < 2 * pairs) {
        k = (j & 1) ? kg_mine + (j >> 1) : (j >> 1);
      } else {
        k = kg_mine > pairs ? j - pairs : j;  // the longer kind's remaining tiles, in order
      }
      return split + static_cast<int64_t>(k) * gridDim.y;
    }
  };

  if (ntiles == 0) {  // nothing to read: an empty partial, or the sink alone
    const int64_t row0 = (static_cast<int64_t>(b) * p.T + t0) * p.H;
    if (p.cluster > 1) {  // an empty share of the cluster's combine (s_m holds -inf)
      if (threadIdx.x < 64) s_l[threadIdx.x] = 0.f;
      stream_cluster_merge(p, s_m, s_l, reinterpret_cast<const float*>(sP), reinterpret_cast<float*>(sK), row0,
                           TQg * p.H);
    } else if (static_cast<int>(threadIdx.x) < NCOL) {
      const int col = threadIdx.x, tq = col / p.H, h = col - tq * p.H;
      if (tq < TQg) {
        const int64_t orow = row0 + tq * p.H + h;
        if (p.splits > 1) {
          p.part_lse[split * rows_total + orow] = -INFINITY;
        } else {
          for (int c = 0; c < C; ++c) p.out[orow * C + c] = __float2bfloat16_rn(0.f);
          p.lse[orow] = p.sink != nullptr ? p.sink[h] : -INFINITY;
        }
      }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
      tc_fence_after();
      tmem_dealloc(*s_tmem, L::TMEM_COLS);
    }
    return;
  }

  const uint32_t tmem = *s_tmem;
  griddep_launch();  // the merge that follows may start launching (it waits for this grid's results)

  if (warp >= 5) {
    // ---------------------------------------------------------- loaders
    const int lt = threadIdx.x - 160;
    const __nv_bfloat16* kb = p.k + static_cast<int64_t>(b) * p.ksb;
    const __nv_bfloat16* vb = p.v + static_cast<int64_t>(b) * p.vsb;
    // range mode: whole 128-row tiles by TMA, one thread, completion by bytes
    auto issue_tile = [&](int j) {
      const int st = j % STAGES;
      const int n0 = range_lo + static_cast<int>((tile0 + j) * BN);
      mbar_expect_tx(full + st, 2 * L::KV_BYTES);
      tma_load_3d(sK + st * L::KV_BYTES, &tm_k, full + st, 0, n0, b);
      tma_load_3d(sK + st * L::KV_BYTES + BN * 128, &tm_k, full + st, 64, n0, b);
      tma_load_3d(sV + st * L::KV_BYTES, &tm_v, full + st, 0, n0, b);
      tma_load_3d(sV + st * L::KV_BYTES + BN * 128, &tm_v, full + st, 64, n0, b);
    };
    if (!GATHER && lt == 0) {  // the first stages need no free slot: in flight together with Q's copy
      for (int j = 0; j < ntiles && j < STAGES; ++j) issue_tile(j);
    }
    // Q: NCOL rows (query x head), zeros for padding columns
    for (int it = lt; it < NCOL * 16; it += STREAM_LOADERS) {
      const int col = it >> 4, ch = it & 15;
      const int tq = col / p.H, h = col - tq * p.H;
      const bool ok = tq < TQg;
      const __nv_bfloat16* src = p.q + ((static_cast<int64_t>(b) * p.T + t0 + tq) * p.H + h) * C + ch * 8;
      cp_async_16(smem_u32(sQ + (ch >> 3) * (NCOL * 128) + sw128_offset(col, ch & 7)), ok ? src : p.q, ok);
    }
    cp_async_commit();
    if constexpr (!GATHER) {
      cp_async_wait<0>();
      fence_proxy_async();
      mbar_arrive(q_full);
      if (lt == 0) {
        for (int j = STAGES; j < ntiles; ++j) {
          if (!mbar_wait(kv_empty + j % STAGES, ((j / STAGES) & 1) ^ 1, p.status)) break;
          issue_tile(j);
        }
      }
      __syncwarp();
    } else {
      const int64_t pos_g = p.positions[static_cast<int64_t>(b) * p.T + t0];
      const int64_t* idx_row = gather ? p.idx + (static_cast<int64_t>(b) * p.T + t0) * p.K : nullptr;
      // A tile is published (full barrier) once this thread's copies for it
      // have landed. Normally tile j - 1 is published right after tile j is
      // issued, keeping two tiles in flight; before blocking on a free stage,
      // every issued tile is published first, since the consumer may need one
      // of them to free that stage.
      // The rows of tile j + 1 are looked up (idx loads in flight) while
      // tile j's copies are in flight.
      auto lookup = [&](int j, int (&rw)[2]) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int64_t slot = tile_of(j) * BN + lt + half * 64;
          int64_t row = -1;
          if (j < ntiles && slot < total) {
            if (!gather) {
              row = range_lo + slot;
            } else if (slot < p.K) {
              row = idx_row[slot];
            } else {
              row = pos_g - p.window + 1 + (slot - p.K);
            }
            if (row < 0 || row >= p.N) row = -1;
          }
          rw[half] = static_cast<int>(row);
        }
      };
      int next_rows[2];
      lookup(0, next_rows);
      bool ok = true;
      int published = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % STAGES;
        if (j >= STAGES) {
          const uint32_t parity = ((j / STAGES) & 1) ^ 1;
          if (!mbar_try_wait(kv_empty + st, parity)) {
            if (published < j) {
              cp_async_wait<0>();
              fence_proxy_async();
              for (; published < j; ++published) mbar_arrive(full + published % STAGES);
            }
            ok = mbar_wait(kv_empty + st, parity, p.status);
          }
        }
        // a failed wait is carried to the barrier below, where the two loader
        // warps agree on it, and the stage's rows are left alone
        int* rows = s_row + st * BN;
        if (ok) {
          rows[lt] = next_rows[0];
          rows[lt + 64] = next_rows[1];
        }
        ok = named_barrier_and(2, STREAM_LOADERS, ok);
        if (!ok) break;
        const uint32_t dk = smem_u32(sK + st * L::KV_BYTES), dv = smem_u32(sV + st * L::KV_BYTES);
        const int64_t first = tile_of(j) * BN;
        if (gather && p.window_tma && first >= p.K) {
          // a tile of window rows is one contiguous range: whole tiles by TMA
          // (rows outside the table read as zeros and are masked)
          if (lt == 0) {
            const int n0 = static_cast<int>(pos_g - p.window + 1 + (first - p.K));
            mbar_expect_tx_only(full + st, 2 * L::KV_BYTES);
            tma_load_3d(sK + st * L::KV_BYTES, &tm_k, full + st, 0, n0, b);
            tma_load_3d(sK + st * L::KV_BYTES + BN * 128, &tm_k, full + st, 64, n0, b);
            tma_load_3d(sV + st * L::KV_BYTES, &tm_v, full + st, 0, n0, b);
            tma_load_3d(sV + st * L::KV_BYTES + BN * 128, &tm_v, full + st, 64, n0, b);
          }
        } else {
#pragma unroll 4
          for (int it = 0; it < (BN * 16) / STREAM_LOADERS; ++it) {
            const int flat = it * STREAM_LOADERS + lt;
            const int r = flat >> 4, ch = flat & 15;
            const int row = rows[r];
            const bool has = row >= 0;
            const uint32_t off = (ch >> 3) * (BN * 128) + sw128_offset(r, ch & 7);
            cp_async_16(dk + off, has ? kb + static_cast<int64_t>(row) * p.ksn + ch * 8 : p.k, has);
            cp_async_16(dv + off, has ? vb + static_cast<int64_t>(row) * p.vsn + ch * 8 : p.v, has);
          }
        }
        cp_async_commit();
        lookup(j + 1, next_rows);
        if (j == 0) {  // Q's copies, the group before tile 0's, were in flight with it
          cp_async_wait<1>();
          fence_proxy_async();
          mbar_arrive(q_full);
        }
        if (published == j - 1) {
          cp_async_wait<1>();
          fence_proxy_async();
          mbar_arrive(full + published % STAGES);
          ++published;
        }
      }
      cp_async_wait<0>();
      fence_proxy_async();
      if (ok) {
        for (; published < ntiles; ++published) mbar_arrive(full + published % STAGES);
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------- MMA issuer
    // the whole warp runs the loop and one elected lane issues; descriptors
    // are warp-uniform bases plus constant offsets
    constexpr uint32_t IDESC_S = idesc_bf16(128, NCOL, 0, 0);
    constexpr uint32_t IDESC_O = idesc_bf16(128, NCOL, 1, 0);
    const uint32_t tS = tmem, tO = tmem + 2 * NCOL;
    const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV), p_addr = smem_u32(sP);
    const uint64_t dq = sdesc_sw128(q_addr, 16, 1024);
    auto wait = [&](uint64_t* bar, int parity) { return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.status)); };
    bool ok = wait(q_full, 0);
    for (int j = 0; ok && j <= ntiles; ++j) {
      if (j < ntiles) {
        const int st = j % STAGES;
        if (!(ok = wait(full + st, (j / STAGES) & 1))) break;
        tc_fence_after();
        stream_s_steps<NCOL, C / 16 - 1>(tS + (j & 1) * NCOL, sdesc_sw128(k_addr + st * L::KV_BYTES, 16, 1024), dq,
                                         IDESC_S);
        mma_commit_warp(s_full + (j & 1));
      }
      if (j > 0) {
        const int jp = j - 1, st = jp % STAGES;
        if (!(ok = wait(p_ready + (jp & 1), (jp >> 1) & 1))) break;
        tc_fence_after();
        stream_pv_steps<NCOL, BN / 16 - 1>(tO, sdesc_sw128(v_addr + st * L::KV_BYTES, BN * 128, 1024),
                                           sdesc_sw128(p_addr + (jp & 1) * L::P_BYTES, 16, 1024), IDESC_O,
                                           jp > 0 ? 1u : 0u);
        mma_commit_warp(kv_empty + st);
        mma_commit_warp(o_done);
        if (j == ntiles) mma_commit_warp(o_final);
      }
    }
  } else {
    // ------------------------------------------ softmax: thread r = slot r
    const int r = threadIdx.x, lane = r & 31;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const uint32_t tO = lane_addr + 2 * NCOL;
    const float sl2 = p.scale_log2;
    float lp[NCOL];
#pragma unroll
    for (int c = 0; c < NCOL; ++c) lp[c] = 0.f;
    // Column masks, read once: column c belongs to query c / H; a tile row
    // is visible to the columns of every query whose bounds contain it.
    const uint64_t head_bits = p.H >= 64 ? ~0ull : ((1ull << p.H) - 1);
    const uint64_t all_cols = TQg * p.H >= 64 ? ~0ull : ((1ull << (TQg * p.H)) - 1);
    int qlo_r[4], qhi_r[4];
#pragma unroll
    for (int tq = 0; tq < 4; ++tq) {
      qlo_r[tq] = tq < TQg ? s_qlo[tq] : 1;
      qhi_r[tq] = tq < TQg ? s_qhi[tq] : 0;
    }
    float mreg[NCOL];  // the columns' running maxima, as s_m holds them
#pragma unroll
    for (int c = 0; c < NCOL; ++c) mreg[c] = -INFINITY;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int st = j % STAGES;
      // a failed wait is carried to the tile's first barrier, where the four warps agree on it
      if constexpr (GATHER) ok = __all_sync(0xffffffffu, mbar_wait(full + st, (j / STAGES) & 1, p.status));
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(s_full + (j & 1), (j >> 1) & 1, p.status));
      tc_fence_after();
      float s[NCOL];
      {
        const uint32_t sa = lane_addr + (j & 1) * NCOL;
        if constexpr (NCOL == 16) {
          uint32_t x[16];
          tmem_ld16(sa, x);
#pragma unroll
          for (int c = 0; c < 16; ++c) s[c] = __uint_as_float(x[c]);
        } else {
#pragma unroll
          for (int c32 = 0; c32 < NCOL / 32; ++c32) {
            uint32_t x[32];
            tmem_ld32(sa + c32 * 32, x);
#pragma unroll
            for (int c = 0; c < 32; ++c) s[c32 * 32 + c] = __uint_as_float(x[c]);
          }
        }
      }
      uint64_t vis;
      if constexpr (GATHER) {
        vis = s_row[st * BN + r] >= 0 ? all_cols : 0ull;
      } else {
        const int row = range_lo + static_cast<int>((tile0 + j) * BN) + r;
        vis = 0ull;
        if (TQg <= 4) {
#pragma unroll
          for (int tq = 0; tq < 4; ++tq)
            if (row >= qlo_r[tq] && row <= qhi_r[tq]) vis |= head_bits << (tq * p.H);
        } else {
          for (int tq = 0; tq < TQg; ++tq)
            if (row >= s_qlo[tq] && row <= s_qhi[tq]) vis |= head_bits << (tq * p.H);
        }
      }
#pragma unroll
      for (int c = 0; c < NCOL; ++c) s[c] = ((vis >> c) & 1ull) ? s[c] * sl2 : -INFINITY;
      // Lazy maximum: a column's running maximum (mreg, the copy of s_m) is
      // raised only when a score exceeds it by more than 8 (base 2), so most
      // tiles need no reduction over their 128 slots: one barrier ORs "some
      // score of mine exceeds its column's maximum + 8" (or "my wait failed")
      // and only then do the maxima, the rescale and the agreement on `ok`
      // run, as below.
      bool raise = false;
#pragma unroll
      for (int c = 0; c < NCOL; ++c) raise |= s[c] > mreg[c] + 8.f;
      float areg[NCOL];
#pragma unroll
      for (int c = 0; c < NCOL; ++c) areg[c] = 1.f;
      bool any = false;
      if (named_barrier_or(1, 128, raise || !ok)) {
        // per-column maximum over the tile's 128 slots
#pragma unroll
        for (int c32 = 0; c32 < (NCOL + 31) / 32; ++c32) {
          float tmp[32];
#pragma unroll
          for (int c = 0; c < 32; ++c) tmp[c] = (c32 * 32 + c < NCOL) ? s[(c32 * 32 + c) % NCOL] : -INFINITY;
          const float m = transpose_reduce32(tmp, MaxOp());
          if (c32 * 32 + lane < NCOL) s_red[warp * 64 + c32 * 32 + lane] = m;
        }
        ok = named_barrier_and(1, 128, ok);
        if (!ok) break;
        if (r < NCOL) {
          const float tmax = fmaxf(fmaxf(s_red[r], s_red[64 + r]), fmaxf(s_red[128 + r], s_red[192 + r]));
          const float mo = s_m[r];
          float a = 1.f;
          if (tmax > mo + 8.f) {
            a = fast_exp2(mo - tmax);
            s_m[r] = tmax;
          }
          s_alpha[r] = a;
        }
        named_barrier(1, 128);
#pragma unroll
        for (int c4 = 0; c4 < NCOL / 4; ++c4) {
          const float4 m4 = reinterpret_cast<const float4*>(s_m)[c4];
          const float4 a4 = reinterpret_cast<const float4*>(s_alpha)[c4];
          mreg[4 * c4] = m4.x;
          mreg[4 * c4 + 1] = m4.y;
          mreg[4 * c4 + 2] = m4.z;
          mreg[4 * c4 + 3] = m4.w;
          areg[4 * c4] = a4.x;
          areg[4 * c4 + 1] = a4.y;
          areg[4 * c4 + 2] = a4.z;
          areg[4 * c4 + 3] = a4.w;
        }
#pragma unroll
        for (int c = 0; c < NCOL; ++c) {
          lp[c] *= areg[c];
          any |= areg[c] != 1.f;
        }
      }
      if (any && j > 0) {  // every thread read the same alphas: uniform
        // (a failed wait skips the rescale; the next tile's barrier stops every warp)
        ok = __all_sync(0xffffffffu, mbar_wait(o_done, (j - 1) & 1, p.status)) && ok;
      }
      if (ok && any && j > 0) {
        tc_fence_after();
        if constexpr (NCOL == 16) {
          uint32_t x[16];
          tmem_ld16(tO, x);
#pragma unroll
          for (int c = 0; c < 16; ++c) x[c] = __float_as_uint(__uint_as_float(x[c]) * areg[c]);
          tmem_st16(tO, x);
        } else {
#pragma unroll
          for (int c32 = 0; c32 < NCOL / 32; ++c32) {
            uint32_t x[32];
            tmem_ld32(tO + c32 * 32, x);
#pragma unroll
            for (int c = 0; c < 32; ++c) x[c] = __float_as_uint(__uint_as_float(x[c]) * areg[c32 * 32 + c]);
            tmem_st32(tO + c32 * 32, x);
          }
        }
      }
      uint8_t* pbuf = sP + (j & 1) * L::P_BYTES + (r >> 6) * (NCOL * 128) + (r & 7) * 2;
      const uint32_t chunk = (r & 63) >> 3;
#pragma unroll
      for (int c = 0; c < NCOL; ++c) {
        const float m = mreg[c];
        const float e = fast_exp2(s[c] - (m == -INFINITY ? 0.f : m));
        lp[c] += e;
        *reinterpret_cast<__nv_bfloat16*>(pbuf + sw128_offset(c, chunk)) = __float2bfloat16_rn(e);
      }
      tmem_wait_st();
      tc_fence_before();
      fence_proxy_async();
      mbar_arrive(p_ready + (j & 1));
    }
    // o_done's parity cannot name the last product here (the MMA may still be
    // two products behind, and phase ntiles - 3 has the same parity), so the
    // epilogue waits on o_final, which completes once, after the last one
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(o_final, 0, p.status));
    tc_fence_after();
    // per-column sums over the 128 slots
#pragma unroll
    for (int c32 = 0; c32 < (NCOL + 31) / 32; ++c32) {
      float tmp[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) tmp[c] = (c32 * 32 + c < NCOL) ? lp[(c32 * 32 + c) % NCOL] : 0.f;
      const float sum = transpose_reduce32(tmp, SumOp());
      if (c32 * 32 + lane < NCOL) s_red[warp * 64 + c32 * 32 + lane] = sum;
    }
    named_barrier(1, 128);
    // thread c < NCOL finishes column c: its normaliser (into s_l) and log-sum
    const int ncols = TQg * p.H;  // columns with a query; the rest are padding
    const int64_t row0 = (static_cast<int64_t>(b) * p.T + t0) * p.H;  // column c is row row0 + c
    if (r < ncols) {
      const float l = (s_red[r] + s_red[64 + r]) + (s_red[128 + r] + s_red[192 + r]);
      const float m = s_m[r], msub = m == -INFINITY ? 0.f : m;
      if (p.cluster > 1) {
        s_l[r] = ok ? l : 0.f;  // combined across the cluster below
      } else if (p.splits == 1) {
        float denom = l;
        if (p.sink != nullptr) denom += fast_exp2(fmaf(p.sink[r % p.H], LOG2E, -msub));
        s_l[r] = denom > 0.f ? 1.f / denom : 0.f;
        if (ok) p.lse[row0 + r] = denom > 0.f ? (msub + log2f(denom)) * LN2 : -INFINITY;
      } else {
        s_l[r] = l > 0.f ? 1.f / l : 0.f;
        if (ok) p.part_lse[split * rows_total + row0 + r] = l > 0.f ? (msub + log2f(l)) * LN2 : -INFINITY;
      }
    }
    named_barrier(1, 128);
    float o[NCOL];
    if (ok) {
      if constexpr (NCOL == 16) {
        uint32_t x[16];
        tmem_ld16(tO, x);
#pragma unroll
        for (int c = 0; c < 16; ++c) o[c] = __uint_as_float(x[c]);
      } else {
#pragma unroll
        for (int c32 = 0; c32 < NCOL / 32; ++c32) {
          uint32_t x[32];
          tmem_ld32(tO + c32 * 32, x);
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c32 * 32 + c] = __uint_as_float(x[c]);
        }
      }
    }
    // thread r holds element r of the head width for every column (query, head)
    if (p.cluster > 1) {
      // unnormalised, into the P buffers (2 x NCOL x 128 bf16 = NCOL x 128
      // floats; the last P V product, which read them, has completed)
      if (ok) {
        float* dst = reinterpret_cast<float*>(sP) + r;
#pragma unroll
        for (int c = 0; c < NCOL; ++c) dst[c * C] = o[c];
      }
    } else if (ok) {
      if (p.splits == 1) {
        __nv_bfloat16* dst = p.out + row0 * C + r;
#pragma unroll
        for (int c = 0; c < NCOL; ++c)
          if (c < ncols) dst[static_cast<int64_t>(c) * C] = __float2bfloat16_rn(o[c] * s_l[c]);
      } else {
        float* dst = p.part_o + (split * rows_total + row0) * C + r;
#pragma unroll
        for (int c = 0; c < NCOL; ++c)
          if (c < ncols) dst[static_cast<int64_t>(c) * C] = o[c] * s_l[c];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
  if (p.cluster > 1)
    stream_cluster_merge(p, s_m, s_l, reinterpret_cast<const float*>(sP), reinterpret_cast<float*>(sK),
                         (static_cast<int64_t>(b) * p.T + t0) * p.H, TQg * p.H);
}

}  // namespace wpt
