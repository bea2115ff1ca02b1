// The long row's combine over NVLink without a collective library: one
// kernel per call on every rank of a long row whose keys are split over the
// GPUs (multi-GPU long-context decode; the reference has no multi-GPU
// inference, so this has no counterpart there).
//
// Every rank holds one exchange buffer, allocated by the library with
// cudaMalloc and mapped into the other ranks' processes with CUDA IPC:
//
//   [0, EXCH_CTRL_BYTES)  control words, uint32:
//       epoch[row]              calls this row's CTA has finished (local only)
//       count[2][row]           arrivals from the ranks, per buffer half
//   then data, fp32:          part[2][world][chunk]
//       chunk = one rank's partial of the call's rows: the output (rows, C),
//       normalised by its softmax sum, then the sum's natural log (rows),
//       padded to 16 bytes
//
// CTA c of every rank takes row c. Per call it
//   1. reads its epoch e (written by the previous call's CTA c, in stream
//      order) and uses buffer half e & 1;
//   2. merges this rank's split partials of its row into one partial (its 8
//      warps share the splits, then combine in shared memory);
//   3. stores that partial into slot `rank` of half e & 1 of EVERY rank's
//      buffer (its own included) with plain stores through the peer
//      mappings (NVLink) and, after a warp barrier, adds 1 to count[e & 1][c]
//      of every rank with a release at system scope;
//   4. waits (bounded: 2 s of %globaltimer, then status bit 0 and no output)
//      until its own count[e & 1][c] reaches world * (e / 2 + 1), i.e. every
//      rank's partial of this call has landed;
//   5. merges the world partials and the sink into out (bf16) and lse;
//   6. sets epoch[c] = e + 1.
// Two halves are enough: a rank can be at most one call ahead of another at
// step 3, since its previous call's step 4 waited for every rank's partial
// of that call, which each rank writes only after finishing the call before.
// The epoch lives in device memory, so a CUDA graph replaying the call
// stays correct. Each rank runs this kernel on its own GPU; the ranks'
// kernels wait for one another, so they must never share a GPU.
#pragma once

#include "common.cuh"

namespace wpt {

constexpr int EXCH_THREADS = 256;    // 8 warps share one row's splits
constexpr int EXCH_BATCH = 4;        // splits a warp loads at once
constexpr int EXCH_MAX_CTAS = 4096;  // one row per CTA, so rows <= 4096
constexpr int64_t EXCH_CTRL_BYTES = 65536;
constexpr int EXCH_MAX_WORLD = 8;

struct ExchangeParams {
  const float* part_o;    // (splits, rows, C) this rank's split partials
  const float* part_lse;  // (splits, rows)
  const float* sink;      // (H,) or null
  uint8_t* peers[EXCH_MAX_WORLD];  // every rank's exchange buffer as mapped here (own at [rank])
  uint8_t* local;         // this rank's buffer
  __nv_bfloat16* out;     // (rows, C)
  float* lse;             // (rows,)
  unsigned* status;
  int64_t chunk;          // floats per rank's partial
  int splits, rows, H, world, rank;
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <int C>
__global__ void __launch_bounds__(EXCH_THREADS) exchange_kernel(const ExchangeParams p) {
  static_assert(C == 128, "each lane moves one float4 of a 128-wide row");
  constexpr int WARPS = EXCH_THREADS / 32;
  griddep_wait();  // the split partials come from the kernel before
  const int row = blockIdx.x;  // CTA c takes row c
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float s_m[WARPS], s_l[WARPS];
  __shared__ float4 s_acc[WARPS][32];
  unsigned* epoch = reinterpret_cast<unsigned*>(p.local);
  const unsigned e = *reinterpret_cast<volatile unsigned*>(epoch + row);
  const int half = static_cast<int>(e & 1u);
  const int64_t slot0 = static_cast<int64_t>(half) * p.world;  // first slot of this half

  // 2. warp w takes splits w, w + 8, ..., EXCH_BATCH at a time with their
  // loads in flight together, in one online pass (running maximum m, sum l
  // and output acc scaled to it); then the warps' results combine
  float m = -INFINITY, l = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = warp; s0 < p.splits; s0 += WARPS * EXCH_BATCH) {
    float lg[EXCH_BATCH];
    float4 v[EXCH_BATCH];
#pragma unroll
    for (int b = 0; b < EXCH_BATCH; ++b) {
      const int sp = s0 + b * WARPS;
      const bool in = sp < p.splits;
      const int64_t r = static_cast<int64_t>(in ? sp : 0) * p.rows + row;
      lg[b] = in ? p.part_lse[r] : -INFINITY;
      v[b] = in ? *reinterpret_cast<const float4*>(p.part_o + r * C + lane * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float nm = m;
#pragma unroll
    for (int b = 0; b < EXCH_BATCH; ++b) nm = fmaxf(nm, lg[b]);
    if (nm == -INFINITY) continue;
    const float sc = __expf(m - nm);  // 0 while m is -inf
    l *= sc;
    acc = make_float4(acc.x * sc, acc.y * sc, acc.z * sc, acc.w * sc);
#pragma unroll
    for (int b = 0; b < EXCH_BATCH; ++b) {
      const float w = __expf(lg[b] - nm);  // 0 for a split with no row
      l += w;
      acc = make_float4(acc.x + w * v[b].x, acc.y + w * v[b].y, acc.z + w * v[b].z, acc.w + w * v[b].w);
    }
    m = nm;
  }
  if (lane == 0) {
    s_m[warp] = m;
    s_l[warp] = l;
  }
  s_acc[warp][lane] = acc;
  __syncthreads();
  if (warp != 0) return;

  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < WARPS; ++w) M = fmaxf(M, s_m[w]);
  float L = 0.f;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  if (M > -INFINITY) {
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      const float sc = __expf(s_m[w] - M);
      const float4 a = s_acc[w][lane];
      L += sc * s_l[w];
      o = make_float4(o.x + sc * a.x, o.y + sc * a.y, o.z + sc * a.z, o.w + sc * a.w);
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  o = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
  const float own_lse = L > 0.f ? M + __logf(L) : -INFINITY;

  // 3. into slot `rank` of every rank's buffer; after the warp's barrier,
  // lane g adds one arrival on rank g with a release at system scope (it
  // orders the warp's stores before the arrival)
  for (int g = 0; g < p.world; ++g) {
    float* dst = reinterpret_cast<float*>(p.peers[g] + EXCH_CTRL_BYTES) + (slot0 + p.rank) * p.chunk;
    *reinterpret_cast<float4*>(dst + static_cast<int64_t>(row) * C + lane * 4) = o;
    if (lane == 0) dst[static_cast<int64_t>(p.rows) * C + row] = own_lse;
  }
  __syncwarp();
  if (lane < p.world)
    red_release_sys_add(reinterpret_cast<unsigned*>(p.peers[lane]) + EXCH_MAX_CTAS * (1 + half) + row, 1u);

  // 4. every rank's partial of this call has landed here
  int ok = 1;
  if (lane == 0) {
    const unsigned* mine = reinterpret_cast<const unsigned*>(p.local) + EXCH_MAX_CTAS * (1 + half) + row;
    const unsigned target = static_cast<unsigned>(p.world) * ((e >> 1) + 1u);
    if (static_cast<int>(ld_acquire_sys(mine) - target) < 0) {
      const unsigned long long start = global_ns();
      for (uint32_t i = 1;; ++i) {
        if (static_cast<int>(ld_acquire_sys(mine) - target) >= 0) break;
        if ((i & 63u) == 0 && global_ns() - start > WAIT_LIMIT_NS) {
          atomicOr(p.status, STATUS_WAIT_TIMEOUT);
          ok = 0;
          break;
        }
      }
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);

  // 5. the ranks' partials and the sink -> out, lse
  if (ok) {
    const float* base = reinterpret_cast<const float*>(p.local + EXCH_CTRL_BYTES) + slot0 * p.chunk;
    const int h = row % p.H;
    float mx = p.sink != nullptr ? p.sink[h] : -INFINITY;
    float lg[EXCH_MAX_WORLD];
    float4 v[EXCH_MAX_WORLD];
#pragma unroll
    for (int g = 0; g < EXCH_MAX_WORLD; ++g) {
      const bool in = g < p.world;
      lg[g] = in ? __ldcg(base + g * p.chunk + static_cast<int64_t>(p.rows) * C + row) : -INFINITY;
      v[g] = in ? __ldcg(reinterpret_cast<const float4*>(base + g * p.chunk + static_cast<int64_t>(row) * C +
                                                         lane * 4))
                : make_float4(0.f, 0.f, 0.f, 0.f);
      mx = fmaxf(mx, lg[g]);
    }
    float den = 0.f;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (mx > -INFINITY) {
      den = p.sink != nullptr ? __expf(p.sink[h] - mx) : 0.f;
#pragma unroll
      for (int g = 0; g < EXCH_MAX_WORLD; ++g) {
        const float w = __expf(lg[g] - mx);  // 0 for none
        den += w;
        a = make_float4(a.x + w * v[g].x, a.y + w * v[g].y, a.z + w * v[g].z, a.w + w * v[g].w);
      }
    }
    const float iv = den > 0.f ? 1.f / den : 0.f;
    __nv_bfloat16* dst = p.out + static_cast<int64_t>(row) * C + lane * 4;
    *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(a.x * iv, a.y * iv);
    *reinterpret_cast<__nv_bfloat162*>(dst + 2) = __floats2bfloat162_rn(a.z * iv, a.w * iv);
    if (lane == 0) p.lse[row] = den > 0.f ? mx + __logf(den) : -INFINITY;
  }

  // 6. this row's calls done (the next call's CTA reads it in stream order)
  if (lane == 0) epoch[row] = e + 1u;
}

}  // namespace wpt
