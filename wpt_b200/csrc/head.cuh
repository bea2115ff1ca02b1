// The output head's product for the writer's sampling step:
// scores (R, V) = h (R, D) W (V, D)^T, bf16 in, fp32 accumulate, on the
// tensor cores with the vocabulary rows as the MMA's M:
//
//   S^T = W h^T    M = 128 vocabulary rows, N = R (rounded up to 16), K = D
//
// so R = 64 decode rows still fill 128-row tiles. Replaces the head call of
// the reference's decode step (packages/wpt-model/src/wpt_model/model.py:
// 267,471: nn.Linear(d_model, vocab, bias=False) under bf16 autocast, whose
// output is bf16 and then widened: the scores are rounded to bf16 here too)
// ahead of its sampling (wpt_inference/__init__.py:173-182, the acceptance
// kernels' statistics and draw).
//
// Persistent: CTA c takes vocabulary tiles c, c + grid, ... Warp 5 loads by
// TMA, for every 64-wide column chunk of D, the tile's W chunk (128 x 128
// bytes) and h's (N x 128 bytes; rows past R read as zeros) into a ring of
// HEAD_STAGES stages; warp 4 issues the products (four K=16 steps a chunk)
// into one of two TMEM accumulators, so that a tile's products run while the
// previous tile's epilogue reads the other; warps 0-3 read their lane
// quadrant (thread = vocabulary row) 32 columns at a time and write its R
// scores (a warp writes 128 contiguous bytes of each score row). N is at
// most 128: larger R are taken 128 rows per launch. The whole grid streams W once
// (268 MB for vocab 65,536 x 2,048): the roofline is HBM. Every mbarrier
// wait is bounded.
#pragma once

#include "common.cuh"

namespace wpt {

constexpr int HEAD_THREADS = 192;  // warps 0-3 epilogue, 4 MMA, 5 loader
constexpr int HEAD_STAGES = 6;

struct HeadParams {
  float* scores;     // (R, V) fp32
  unsigned* status;
  int R, V, D, tiles;
  int round_bf16;    // 1: each score rounded to bf16 (the reference's autocast output), then widened
};

template <int N>
struct HeadLayout {
  static constexpr int W_BYTES = 128 * 128;  // one 64-column chunk of a vocabulary tile
  static constexpr int H_BYTES = N * 128;    // the same chunk of h
  static constexpr int STAGE_BYTES = W_BYTES + H_BYTES;
  static constexpr int OFF_BAR = HEAD_STAGES * STAGE_BYTES;
  // full[STAGES], empty[STAGES], acc_full[2], acc_empty[2]
  static constexpr int NBAR = 2 * HEAD_STAGES + 4;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16 + 1024;
  static constexpr int TMEM_COLS = 2 * N <= 32 ? 32 : 2 * N <= 64 ? 64 : 2 * N <= 128 ? 128 : 2 * N <= 256 ? 256 : 512;
};

// S^T (+)= W_chunk h_chunk^T over the chunk's four K=16 steps.
template <int KK>
__device__ __forceinline__ void head_steps(uint32_t d, uint64_t dw, uint64_t dh, uint32_t idesc, uint32_t acc0) {
  if constexpr (KK > 0) head_steps<KK - 1>(d, dw, dh, idesc, acc0);
  constexpr uint32_t off = (KK * 32) >> 4;
  mma_ss_off_warp<off, off>(d, dw, dh, idesc, KK > 0 ? 1u : acc0);
}

template <int N>
__global__ void __launch_bounds__(HEAD_THREADS, 1)
    head_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_h,
                const HeadParams p) {
  using L = HeadLayout<N>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = full + HEAD_STAGES;
  uint64_t* acc_full = empty + HEAD_STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = p.D / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < HEAD_STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(acc_full + s, 1);
      mbar_init(acc_empty + s, 128);
    }
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(s_tmem, L::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 5 && lane == 0) {
    tma_prefetch(&tm_w);
    tma_prefetch(&tm_h);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 5) {
    // ------------------------------------------------------------ loader
    if (lane == 0) {
      bool ok = true;
      int u = 0;  // ring entries issued
      for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x) {
        for (int c = 0; ok && c < chunks; ++c, ++u) {
          const int st = u % HEAD_STAGES;
          if (u >= HEAD_STAGES && !(ok = mbar_wait(empty + st, ((u / HEAD_STAGES) & 1) ^ 1, p.status))) break;
          uint8_t* stage = smem + st * L::STAGE_BYTES;
          mbar_expect_tx(full + st, L::STAGE_BYTES);
          tma_load_2d(stage, &tm_w, full + st, c * 64, t * 128);
          tma_load_2d(stage + L::W_BYTES, &tm_h, full + st, c * 64, 0);
        }
      }
    }
    __syncwarp();
  } else if (warp == 4) {
    // ------------------------------------------------------- MMA issuer
    constexpr uint32_t IDESC = idesc_bf16(128, N, 0, 0);
    auto wait = [&](uint64_t* bar, int parity) { return __all_sync(0xffffffffu, mbar_wait(bar, parity, p.status)); };
    bool ok = true;
    int u = 0, i = 0;  // ring entries consumed, tiles done
    for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x, ++i) {
      const int buf = i & 1;
      // the epilogue has read this accumulator's previous tile
      if (i >= 2 && !(ok = wait(acc_empty + buf, ((i >> 1) & 1) ^ 1))) break;
      tc_fence_after();
      const uint32_t d = tmem + buf * N;
      for (int c = 0; c < chunks; ++c, ++u) {
        const int st = u % HEAD_STAGES;
        if (!(ok = wait(full + st, (u / HEAD_STAGES) & 1))) break;
        tc_fence_after();
        const uint32_t a = smem_u32(smem + st * L::STAGE_BYTES);
        head_steps<3>(d, sdesc_sw128(a, 16, 1024), sdesc_sw128(a + L::W_BYTES, 16, 1024), IDESC, c > 0 ? 1u : 0u);
        mma_commit_warp(empty + st);
      }
      if (ok) mma_commit_warp(acc_full + buf);
    }
  } else {
    // ----------------------------------------------------------- epilogue
    const int row = warp * 32 + lane;  // the tile's vocabulary row this thread owns
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    bool ok = true;
    int i = 0;
    for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x, ++i) {
      const int buf = i & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(acc_full + buf, (i >> 1) & 1, p.status));
      if (!ok) break;
      tc_fence_after();
      // 32 (or 16) columns at a time: each warp writes 128 contiguous bytes of a score row
      const int v = t * 128 + row;
#pragma unroll
      for (int c0 = 0; c0 < N; c0 += 32) {
        uint32_t x[32];
        if (c0 + 32 <= N) {
          tmem_ld32(lane_addr + buf * N + c0, x);
        } else {
          tmem_ld16(lane_addr + buf * N + c0, *reinterpret_cast<uint32_t(*)[16]>(x));
        }
        if (v < p.V) {
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            const int r = c0 + k;
            if (r < N && r < p.R) {
              float s = __uint_as_float(x[k]);
              if (p.round_bf16) s = __bfloat162float(__float2bfloat16_rn(s));
              p.scores[static_cast<int64_t>(r) * p.V + v] = s;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(acc_empty + buf);  // the accumulator may take the tile after next
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

}  // namespace wpt
