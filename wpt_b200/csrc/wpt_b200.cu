// The one translation unit of libwpt_b200.so: the kernels (headers beside
// this file) and the extern "C" launchers declared in include/wpt_attn.h.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>
#include <string>

#include "../../include/wpt_attn.h"
#include "accept.cuh"
#include "backward.cuh"
#include "cache.cuh"
#include "common.cuh"
#include "exchange.cuh"
#include "head.cuh"
#include "merge.cuh"
#include "prefill.cuh"
#include "select.cuh"
#include "stream.cuh"
#include "tree.cuh"

namespace {

thread_local std::string g_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(WPT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

__device__ unsigned g_status_word;

// One lock for every per-device cache of a device symbol's address (the
// status word here, the no-alloc scratch below). The caches are filled once
// per device and never refreshed: the library must not be used across a
// cudaDeviceReset (or any teardown of the device's primary context), after
// which the cached addresses would be stale.
std::mutex g_symbol_lock;

// The device address of the status word on the current device.
int status_word(unsigned** out) {
  static unsigned* cached[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(WPT_ERR_INVALID, "device %d out of range", dev);
  std::lock_guard<std::mutex> guard(g_symbol_lock);
  if (cached[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_status_word);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status)");
    cached[dev] = static_cast<unsigned*>(p);
  }
  *out = cached[dev];
  return WPT_OK;
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encoder(EncodeTiled* out) {
  static EncodeTiled fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr)
      return fail(WPT_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    fn = reinterpret_cast<EncodeTiled>(p);
  }
  *out = fn;
  return WPT_OK;
}

// A bf16 tensor map with 128-byte swizzle and 64-element inner boxes.
// Makes the current device's primary context current on this host thread.
// Runtime calls bind it lazily, but the driver's tensor-map encoder needs it
// bound already, and a thread that has made no runtime call on the device
// yet (autograd's backward worker, for one) has none: cudaSetDevice binds it.
// Once per thread and device.
int bind_context() {
  static thread_local int bound = -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (bound != dev) {
    e = cudaSetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    bound = dev;
  }
  return WPT_OK;
}

// A tensor map depends only on its base address, shape, strides and box, so
// each host thread keeps its last few encodings and a repeated call (a
// decode loop over the same tables) skips the driver's encoder.
struct MapKey {
  const void* base;
  int rank, dev;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3];
};

int tensor_map_encode(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
                      const cuuint64_t* strides_bytes, const cuuint32_t* box);
int current_device(int* sms = nullptr);

int tensor_map(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
               const cuuint32_t* box) {
  constexpr int SLOTS = 16;
  static thread_local MapKey keys[SLOTS];
  static thread_local CUtensorMap maps[SLOTS];
  static thread_local int used = 0, next = 0;
  MapKey key;
  memset(&key, 0, sizeof(key));
  key.base = base;
  key.rank = rank;
  key.dev = current_device();
  for (int i = 0; i < rank; ++i) {
    key.dims[i] = dims[i];
    key.box[i] = box[i];
    if (i + 1 < rank) key.strides[i] = strides_bytes[i];
  }
  for (int i = 0; i < used; ++i)
    if (memcmp(&keys[i], &key, sizeof(key)) == 0) {
      *map = maps[i];
      return WPT_OK;
    }
  if (int rc = tensor_map_encode(map, base, rank, dims, strides_bytes, box)) return rc;
  keys[next] = key;
  maps[next] = *map;
  next = (next + 1) % SLOTS;
  if (used < SLOTS) ++used;
  return WPT_OK;
}

int tensor_map_encode(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
                      const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  EncodeTiled encode;
  if (int rc = encoder(&encode)) return rc;
  if (int rc = bind_context()) return rc;
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides_bytes,
                      box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(WPT_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return WPT_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// A (B, N, C) table as a 3-D map {C, N, B} with boxes of {64, 128, 1}.
int table_map(CUtensorMap* map, const void* base, int64_t stride_b, int64_t stride_n, int B, int N, int C) {
  if (!aligned16(base)) return fail(WPT_ERR_INVALID, "a key/value table is not 16-byte aligned");
  if (stride_n % 8 != 0 || (B > 1 && stride_b % 8 != 0) || stride_n < C)
    return fail(WPT_ERR_INVALID, "key/value strides must be multiples of 8 elements (got %lld, %lld)",
                static_cast<long long>(stride_b), static_cast<long long>(stride_n));
  if (B == 1) stride_b = static_cast<int64_t>(N) * stride_n;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(stride_n) * 2, static_cast<cuuint64_t>(stride_b) * 2};
  cuuint32_t box[3] = {64, 128, 1};
  return tensor_map(map, base, 3, dims, strides, box);
}

// The current device (and its SM count), asked of the runtime once per
// thread and device change rather than on every launch.
int current_device(int* sms) {
  static thread_local int cached_sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (sms) {
    if (cached_sms[dev] == 0) {
      int v = 148;
      if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) v = 148;
      cached_sms[dev] = v;
    }
    *sms = cached_sms[dev];
  }
  return dev;
}

// Raises a kernel's dynamic shared memory limit to `bytes` on the current
// device, once per (kernel, device, size): the attribute call costs
// microseconds that a decode step should not pay on every launch.
template <typename Kernel>
int allow_smem(Kernel kernel, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;
  const int dev = current_device();
  const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = done.find(key);
    if (it != done.end() && it->second >= bytes) return WPT_OK;
  }
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic shared memory)");
  std::lock_guard<std::mutex> lock(mu);
  done[key] = bytes;
  return WPT_OK;
}

// Q-pair buffers and K/V ring stages of the prefill kernel: the ring gets
// what 227 KB leaves after the Q buffers (the next item's Q is prefetched
// into L2 instead of a second buffer when C = 128).
template <int C>
struct PrefillShape {
  static constexpr int QB = C == 128 ? 1 : 2, NS = C == 128 ? 5 : 8;
};

// Pairs of weights in every 8 computed on the FMA pipe (WPT_B200_POLY8 = 0..4 overrides).
int prefill_poly8() {
  static int v = -1;
  if (v < 0) {
    const char* env = getenv("WPT_B200_POLY8");
    const int e = env ? atoi(env) : 1;
    v = (e >= 0 && e <= 4) ? e : 1;
  }
  return v;
}

template <int C, int POLY8, bool CLUSTER>
int launch_prefill_p(const wpt::PrefillParams& p, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                     const CUtensorMap& to, cudaStream_t stream) {
  constexpr int QB = PrefillShape<C>::QB, NS = PrefillShape<C>::NS;
  using L = wpt::PrefillLayout<C, QB, NS>;
  static_assert(L::BYTES <= 232448, "prefill kernel shared memory exceeds 227 KB");
  auto kernel = wpt::prefill_kernel<C, QB, NS, POLY8, CLUSTER>;
  if (int rc = allow_smem(kernel, L::BYTES)) return rc;
  // setmaxnreg redistributes the registers the block was launched with: a
  // kernel built with fewer than REGS_LAUNCH would leave the softmax
  // warpgroups' increase waiting forever, so it is refused here instead
  static int regs = -1;
  if (regs < 0) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes(prefill_kernel)");
    regs = fa.numRegs;
  }
  if (regs != L::REGS_LAUNCH)
    return fail(WPT_ERR_CUDA, "prefill_kernel built with %d registers a thread, its register split needs %d", regs,
                L::REGS_LAUNCH);
  int sms = 148;
  current_device(&sms);
  const int grid = p.items < sms ? p.items : sms;  // persistent: one CTA per SM walks the items
  if (p.cluster && (grid != p.items || p.items % 2 != 0))
    return fail(WPT_ERR_INVALID, "prefill cluster mode needs one item per CTA (%d items, %d SMs)", p.items, sms);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;  // cluster mode: a pair's two splits per cluster
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.cluster ? 1 : 0;
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(L::THREADS);
  cfg.dynamicSmemBytes = L::BYTES;
  cfg.stream = stream;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tq, tk, tv, to, p);
  if (e != cudaSuccess) return cuda_fail(e, "prefill_kernel launch");
  return WPT_OK;
}

template <int C>
int launch_prefill(const wpt::PrefillParams& p, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                   const CUtensorMap& to,
                   cudaStream_t stream) {
  // the cluster-combine instance (the POLY8 overrides are for sweeps of the plain one)
  if (p.cluster) return launch_prefill_p<C, 1, true>(p, tq, tk, tv, to, stream);
  switch (prefill_poly8()) {
    case 0: return launch_prefill_p<C, 0, false>(p, tq, tk, tv, to, stream);
    case 3: return launch_prefill_p<C, 3, false>(p, tq, tk, tv, to, stream);
    case 4: return launch_prefill_p<C, 4, false>(p, tq, tk, tv, to, stream);
    case 2: return launch_prefill_p<C, 2, false>(p, tq, tk, tv, to, stream);
    default: return launch_prefill_p<C, 1, false>(p, tq, tk, tv, to, stream);
  }
}

// 1: the key-stream kernel launches as a programmatic dependent of the
// kernel before it on the stream (WPT_B200_PDL = 0 or 1 overrides).
int stream_pdl() {
  static int v = -1;
  if (v < 0) {
    const char* env = getenv("WPT_B200_PDL");
    v = env ? (atoi(env) != 0) : 1;
  }
  return v;
}

template <int NCOL, int STAGES, bool GATHER>
int launch_stream_n(const CUtensorMap& tk, const CUtensorMap& tv, const wpt::StreamParams& p, int groups,
                    cudaStream_t stream) {
  using L = wpt::StreamLayout<NCOL, STAGES>;
  static_assert(L::BYTES <= 232448, "key-stream kernel shared memory exceeds 227 KB");
  auto kernel = wpt::stream_kernel<NCOL, STAGES, GATHER>;
  if (int rc = allow_smem(kernel, L::BYTES)) return rc;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (stream_pdl()) {  // its set-up overlaps the tail of the kernel before it (it waits on the device)
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na++].val.programmaticStreamSerializationAllowed = 1;
  }
  if (p.cluster > 1) {  // cluster mode: one group's splits per cluster
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = p.cluster;
    attr[na++].val.clusterDim.z = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cfg.gridDim = dim3(groups, p.splits);
  cfg.blockDim = dim3(wpt::STREAM_THREADS);
  cfg.dynamicSmemBytes = L::BYTES;
  cfg.stream = stream;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tk, tv, p);
  if (e != cudaSuccess) return cuda_fail(e, "stream_kernel launch");
  return WPT_OK;
}

template <bool GATHER>
int launch_stream_g(const CUtensorMap& tk, const CUtensorMap& tv, const wpt::StreamParams& p, int ncol, int groups,
                    cudaStream_t stream) {
  switch (ncol) {
    case 16: return launch_stream_n<16, 3, GATHER>(tk, tv, p, groups, stream);
    case 32: return launch_stream_n<32, 3, GATHER>(tk, tv, p, groups, stream);
    default: return launch_stream_n<64, 2, GATHER>(tk, tv, p, groups, stream);
  }
}

template <int NCOL>
int launch_score(const CUtensorMap& tq, const CUtensorMap& tk, const wpt::ScoreParams& p, int groups, int splits,
                 cudaStream_t stream) {
  constexpr int STAGES = 4;
  using L = wpt::ScoreLayout<NCOL, STAGES>;
  static_assert(L::BYTES <= 232448, "score kernel shared memory exceeds 227 KB");
  auto kernel = wpt::score_kernel<NCOL, STAGES>;
  if (int rc = allow_smem(kernel, L::BYTES)) return rc;
  int sms = 148;
  current_device(&sms);
  const dim3 grid = p.balanced ? dim3(sms) : dim3(groups, splits);  // balanced: one CTA per SM
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // waits for lse on the device
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = grid;
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = L::BYTES;
  cfg.stream = stream;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tq, tk, p);
  if (e != cudaSuccess) return cuda_fail(e, "score_kernel launch");
  return WPT_OK;
}

template <int C>
// pdl: the merge directly follows the attention kernel that wrote the
// partials, and launches while that kernel finishes (programmatic dependent
// launch; the merge waits for it on the device before reading).
int launch_merge(const float* part_o, const float* part_lse, int splits, int64_t rows, wpt::SplitLayout lay, int H,
                 const float* sink, void* out, float* lse, cudaStream_t stream, bool pdl = false,
                 float* out_f32 = nullptr) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cfg.stream = stream;
  cfg.dynamicSmemBytes = 0;
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
  cudaError_t e;
  if (splits >= 16 && splits <= wpt::MERGE_MAX_SPLITS && rows <= 4096) {  // few rows, many splits: a CTA per row
    cfg.gridDim = dim3(static_cast<unsigned>(rows));
    cfg.blockDim = dim3(wpt::MERGE_THREADS);
    e = cudaLaunchKernelEx(&cfg, wpt::merge_wide_kernel<C>, part_o, part_lse, splits, lay, H, sink, o, lse, out_f32);
  } else {
    const int warps = 8;
    const int64_t blocks = (rows + warps - 1) / warps;
    cfg.gridDim = dim3(static_cast<unsigned>(blocks));
    cfg.blockDim = dim3(warps * 32);
    e = cudaLaunchKernelEx(&cfg, wpt::merge_kernel<C>, part_o, part_lse, splits, rows, lay, H, sink, o, lse,
                           out_f32);
  }
  if (e != cudaSuccess) return cuda_fail(e, "merge_kernel launch");
  return WPT_OK;
}

// The plain (splits, rows) layout at split stride `split_stride` rows.
template <int C>
int launch_merge(const float* part_o, const float* part_lse, int splits, int64_t rows, int64_t split_stride, int H,
                 const float* sink, void* out, float* lse, cudaStream_t stream, bool pdl = false) {
  wpt::SplitLayout lay;
  lay.per = splits;
  lay.stride = split_stride;
  lay.group_o = 0;
  lay.group_l = 0;
  return launch_merge<C>(part_o, part_lse, splits, rows, lay, H, sink, out, lse, stream, pdl);
}

}  // namespace

extern "C" const char* wpt_last_error(void) { return g_error.c_str(); }

extern "C" int wpt_status(unsigned* status, int reset) {
  unsigned* word = nullptr;
  if (int rc = status_word(&word)) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  unsigned value = 0;
  e = cudaMemcpy(&value, word, sizeof(value), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read status");
  if (reset) {
    e = cudaMemset(word, 0, sizeof(unsigned));
    if (e != cudaSuccess) return cuda_fail(e, "reset status");
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  }
  if (status) *status = value;
  return WPT_OK;
}

extern "C" int wpt_attn_prefill(const void* q, const void* k, const void* v, int64_t k_stride_b, int64_t k_stride_n,
                                int64_t v_stride_b, int64_t v_stride_n, const int64_t* positions,
                                const int64_t* floor_rows, const uint64_t* tree_bits, const int64_t* tree_base,
                                const float* sink, void* out, float* lse, float* part_o, float* part_lse, int splits,
                                int B, int T, int H, int C, int N, int window, float scale, void* stream) {
  if (C != 64 && C != 128) return fail(WPT_ERR_UNSUPPORTED, "head width %d: the kernels take 64 or 128", C);
  if (H < 1 || H > 128) return fail(WPT_ERR_UNSUPPORTED, "%d heads: the kernels take 1 to 128", H);
  if (B < 1 || T < 1 || N < 1) return fail(WPT_ERR_INVALID, "empty shape B=%d T=%d N=%d", B, T, N);
  if (static_cast<int64_t>(B) * T * H + 256 >= (int64_t(1) << 31)) return fail(WPT_ERR_UNSUPPORTED, "B*T*H too large");
  if (splits < 1) return fail(WPT_ERR_INVALID, "splits must be >= 1");
  // part_o and part_lse both NULL with 2 splits: cluster mode (a pair's two
  // splits combine in shared memory; no scratch, no merge launch)
  const bool cluster = splits == 2 && part_o == nullptr && part_lse == nullptr;
  if (splits > 1 && !cluster && (part_o == nullptr || part_lse == nullptr))
    return fail(WPT_ERR_INVALID, "splits > 1 needs part_o and part_lse scratch (or neither, for 2)");
  if (tree_bits != nullptr && tree_base == nullptr) return fail(WPT_ERR_INVALID, "tree_bits needs tree_base");
  if (!q || !k || !v || !positions || !out || !lse) return fail(WPT_ERR_INVALID, "a required pointer is NULL");
  if (!aligned16(q) || !aligned16(out)) return fail(WPT_ERR_INVALID, "q and out must be 16-byte aligned");
  if (!(scale > 0.f)) return fail(WPT_ERR_INVALID, "scale must be positive");

  CUtensorMap tq, tk, tv, to;  // to: the output, same shape as q (full query tiles leave by TMA store)
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(B) * T * H};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(C) * 2};
    cuuint32_t box[2] = {64, 128};
    if (int rc = tensor_map(&tq, q, 2, dims, strides, box)) return rc;
    if (int rc = tensor_map(&to, out, 2, dims, strides, box)) return rc;
  }
  if (int rc = table_map(&tk, k, k_stride_b, k_stride_n, B, N, C)) return rc;
  if (int rc = table_map(&tv, v, v_stride_b, v_stride_n, B, N, C)) return rc;

  wpt::PrefillParams p;
  p.positions = positions;
  p.floor_rows = floor_rows;
  p.tree_bits = tree_bits;
  p.tree_base = tree_base;
  p.sink = splits > 1 && !cluster ? nullptr : sink;  // cluster mode: its combine adds the sink
  p.cluster = cluster ? 1 : 0;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.lse = lse;
  p.part_o = part_o;
  p.part_lse = part_lse;
  p.tma_out = splits > 1 ? 0 : 1;
  if (int rc = status_word(&p.status)) return rc;
  p.B = B;
  p.T = T;
  p.H = H;
  p.N = N;
  p.window = window > 0 ? window : 0;
  p.TQ = 128 / H;
  p.splits = splits;
  {
    const int64_t items = static_cast<int64_t>((T + 2 * p.TQ - 1) / (2 * p.TQ)) * B * splits;  // query-tile pairs
    if (items >= (int64_t(1) << 31)) return fail(WPT_ERR_UNSUPPORTED, "too many prefill work items");
    p.items = static_cast<int>(items);
  }
  p.scale_log2 = scale * wpt::LOG2E;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = C == 128 ? launch_prefill<128>(p, tq, tk, tv, to, s) : launch_prefill<64>(p, tq, tk, tv, to, s);
  if (rc) return rc;
  if (splits > 1 && !cluster) {
    const int64_t rows = static_cast<int64_t>(B) * T * H;
    rc = C == 128 ? launch_merge<128>(part_o, part_lse, splits, rows, rows, H, sink, out, lse, s, true)
                  : launch_merge<64>(part_o, part_lse, splits, rows, rows, H, sink, out, lse, s, true);
  }
  return rc;
}

// ---------------------------------------------------------------- backward
namespace {

struct BwdScratch {
  int64_t ld, ranges, bounds, sink_part, kv_part, total;  // byte offsets, each 256-aligned
  int kv_parts;
};

// Parts per key tile of the key-tile kernel: enough CTAs for about two per
// SM, since under a causal mask key tile 0 is read by every query tile and
// the last one by a few, and the most-read tile sets the kernel's length.
int bwd_kv_parts(int B, int N) {
  int sms = 148;
  current_device(&sms);
  const int64_t units = static_cast<int64_t>(B) * ((N + 127) / 128);
  const int64_t want = (2 * static_cast<int64_t>(sms) + units - 1) / units;
  return static_cast<int>(want < 1 ? 1 : want > 8 ? 8 : want);
}

BwdScratch bwd_scratch(int B, int T, int H, int N) {
  const int TQ = 128 / H;
  const int64_t qtiles = (T + TQ - 1) / TQ;
  auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
  BwdScratch s;
  s.kv_parts = bwd_kv_parts(B, N);
  s.ld = 0;
  s.ranges = s.ld + up(static_cast<int64_t>(B) * qtiles * 256 * 4);
  s.bounds = s.ranges + up(static_cast<int64_t>(B) * qtiles * 8);
  s.sink_part = s.bounds + up(static_cast<int64_t>(B) * T * 8);
  s.kv_part = s.sink_part + up(static_cast<int64_t>(B) * qtiles * H * 4);
  s.total = s.kv_part + (s.kv_parts > 1 ? up(static_cast<int64_t>(s.kv_parts) * B * N * 256 * 4) : 0);
  return s;
}

}  // namespace

// The failure-detection test hook of wpt_debug_backward_fault.
std::atomic<int> g_bwd_skip_key_tile{-1};
std::atomic<unsigned long long> g_bwd_wait_ns{0};

extern "C" int wpt_debug_backward_fault(int skip_key_tile, unsigned long long wait_ns) {
  if (skip_key_tile < -1) return fail(WPT_ERR_INVALID, "skip_key_tile must be -1 (off) or a key tile index");
  g_bwd_skip_key_tile.store(skip_key_tile);
  g_bwd_wait_ns.store(wait_ns);
  return WPT_OK;
}

extern "C" size_t wpt_attn_backward_scratch_bytes(int B, int T, int H, int C, int N) {
  if (B < 1 || T < 1 || H < 1 || H > 128 || C != 128 || N < 1) return 0;
  return static_cast<size_t>(bwd_scratch(B, T, H, N).total);
}

template <int NCOL>
int launch_gather_bwd(const wpt::GatherBwdParams& g, cudaStream_t st) {
  using L = wpt::GatherBwdLayout<NCOL>;
  static_assert(L::BYTES <= 232448, "gathered-rows backward shared memory exceeds 227 KB");
  if (int rc = allow_smem(wpt::bwd_gather_kernel<NCOL>, L::BYTES)) return rc;
  wpt::bwd_gather_kernel<NCOL><<<static_cast<unsigned>(static_cast<int64_t>(g.B) * g.T), wpt::GBWD_THREADS, L::BYTES,
                                 st>>>(g);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bwd_gather_kernel launch");
  return WPT_OK;
}

extern "C" int wpt_attn_backward(const void* q, const void* k, const void* v, int64_t k_stride_b, int64_t k_stride_n,
                                 int64_t v_stride_b, int64_t v_stride_n, const int64_t* positions,
                                 const int64_t* floor_rows, const int64_t* idx, int K, const float* sink,
                                 const void* out, const float* lse, const void* d_out, void* dq, void* dk, void* dv,
                                 float* d_sink, void* scratch, int f32_grads, int B, int T, int H, int C, int N,
                                 int window, float scale, void* stream) {
  if (K < 0 || (K > 0 && idx == nullptr)) return fail(WPT_ERR_INVALID, "K=%d chosen rows need idx", K);
  if (K > 0 && !f32_grads)
    return fail(WPT_ERR_INVALID, "gradients over chosen rows accumulate in fp32: pass f32_grads = 1");
  if (K > 0 && H > 64) return fail(WPT_ERR_UNSUPPORTED, "%d heads: the gathered-rows backward takes up to 64", H);
  if (C != 128) return fail(WPT_ERR_UNSUPPORTED, "head width %d: the backward kernels take 128", C);
  if (H < 1 || H > 128) return fail(WPT_ERR_UNSUPPORTED, "%d heads: the kernels take 1 to 128", H);
  if (B < 1 || T < 1 || N < 1) return fail(WPT_ERR_INVALID, "empty shape B=%d T=%d N=%d", B, T, N);
  if (static_cast<int64_t>(B) * T * H + 256 >= (int64_t(1) << 31)) return fail(WPT_ERR_UNSUPPORTED, "B*T*H too large");
  if (static_cast<int64_t>(B) * N * C >= (int64_t(1) << 40)) return fail(WPT_ERR_UNSUPPORTED, "B*N too large");
  if (!q || !k || !v || !positions || !out || !lse || !d_out || !dq || !dk || !dv || !scratch)
    return fail(WPT_ERR_INVALID, "a required pointer is NULL");
  if (!aligned16(q) || !aligned16(out) || !aligned16(d_out) || !aligned16(dq) || !aligned16(dk) || !aligned16(dv) ||
      !aligned16(scratch))
    return fail(WPT_ERR_INVALID, "q, out, d_out, dq, dk, dv and scratch must be 16-byte aligned");
  if (sink == nullptr && d_sink != nullptr) return fail(WPT_ERR_INVALID, "d_sink needs sink");
  if (!(scale > 0.f)) return fail(WPT_ERR_INVALID, "scale must be positive");
  CUtensorMap tq, tdo, tk, tv;
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(B) * T * H};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(C) * 2};
    cuuint32_t box[2] = {64, 128};
    if (int rc = tensor_map(&tq, q, 2, dims, strides, box)) return rc;
    if (int rc = tensor_map(&tdo, d_out, 2, dims, strides, box)) return rc;
  }
  if (int rc = table_map(&tk, k, k_stride_b, k_stride_n, B, N, C)) return rc;
  if (int rc = table_map(&tv, v, v_stride_b, v_stride_n, B, N, C)) return rc;
  const BwdScratch lay = bwd_scratch(B, T, H, N);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  wpt::BwdParams p;
  p.positions = positions;
  p.floor_rows = floor_rows;
  p.out = static_cast<const __nv_bfloat16*>(out);
  p.d_out = static_cast<const __nv_bfloat16*>(d_out);
  p.lse = lse;
  p.sink = sink;
  p.ld = reinterpret_cast<float*>(base + lay.ld);
  p.ranges = reinterpret_cast<int2*>(base + lay.ranges);
  p.bounds = reinterpret_cast<int2*>(base + lay.bounds);
  p.sink_part = reinterpret_cast<float*>(base + lay.sink_part);
  p.dq = dq;
  p.dk = dk;
  p.dv = dv;
  p.d_sink = d_sink;
  if (int rc = status_word(&p.status)) return rc;
  p.B = B;
  p.T = T;
  p.H = H;
  p.N = N;
  p.window = window > 0 ? window : 0;
  p.TQ = 128 / H;
  p.qtiles = (T + p.TQ - 1) / p.TQ;
  p.ktiles = (N + 127) / 128;
  p.f32_grads = f32_grads ? 1 : 0;
  p.scale = scale;
  p.scale_log2 = scale * wpt::LOG2E;
  p.kv_parts = lay.kv_parts;
  p.kv_part = reinterpret_cast<float*>(base + lay.kv_part);
  p.skip_key_tile = g_bwd_skip_key_tile.load();
  p.wait_ns = g_bwd_wait_ns.load();
  if (p.wait_ns == 0) p.wait_ns = wpt::WAIT_LIMIT_NS;
  if (static_cast<int64_t>(p.qtiles) * B >= (int64_t(1) << 31) ||
      static_cast<int64_t>(p.ktiles) * B * p.kv_parts >= (int64_t(1) << 31) || B > 65535)
    return fail(WPT_ERR_UNSUPPORTED, "backward grid too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  wpt::bwd_prep_kernel<<<dim3(p.qtiles, B), 128, 0, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bwd_prep_kernel launch");
  if (d_sink != nullptr) {
    wpt::bwd_sink_kernel<<<H, 256, 0, st>>>(p.sink_part, static_cast<int64_t>(B) * p.qtiles, H, d_sink);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "bwd_sink_kernel launch");
  }
  static_assert(wpt::BwdKvLayout::BYTES <= 232448, "backward key kernel shared memory exceeds 227 KB");
  static_assert(wpt::BwdQLayout::BYTES <= 232448, "backward query kernel shared memory exceeds 227 KB");
  if (int rc = allow_smem(wpt::bwd_kv_kernel, wpt::BwdKvLayout::BYTES)) return rc;
  if (int rc = allow_smem(wpt::bwd_q_kernel, wpt::BwdQLayout::BYTES)) return rc;
  wpt::bwd_kv_kernel<<<static_cast<unsigned>(static_cast<int64_t>(p.ktiles) * B * p.kv_parts), wpt::BWD_THREADS,
                       wpt::BwdKvLayout::BYTES, st>>>(tq, tdo, tk, tv, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bwd_kv_kernel launch");
  if (p.kv_parts > 1) {
    int sms = 148;
    current_device(&sms);
    const int64_t n4 = static_cast<int64_t>(B) * N * 64;
    const int blocks = static_cast<int>(std::min<int64_t>((n4 + 255) / 256, static_cast<int64_t>(sms) * 8));
    wpt::bwd_kv_reduce_kernel<<<blocks, 256, 0, st>>>(p.kv_part, p.kv_parts, static_cast<int64_t>(B) * N, dk, dv,
                                                      p.f32_grads);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "bwd_kv_reduce_kernel launch");
  }
  wpt::bwd_q_kernel<<<static_cast<unsigned>(p.qtiles * B), wpt::BWD_THREADS, wpt::BwdQLayout::BYTES, st>>>(
      tq, tdo, tk, tv, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "bwd_q_kernel launch");
  if (K > 0) {  // the chosen rows' share, added to the fp32 gradients above
    wpt::GatherBwdParams g;
    g.q = static_cast<const __nv_bfloat16*>(q);
    g.d_out = static_cast<const __nv_bfloat16*>(d_out);
    g.k = static_cast<const __nv_bfloat16*>(k);
    g.v = static_cast<const __nv_bfloat16*>(v);
    g.ksb = k_stride_b;
    g.ksn = k_stride_n;
    g.vsb = v_stride_b;
    g.vsn = v_stride_n;
    g.idx = idx;
    g.ld = p.ld;
    g.dq = static_cast<float*>(dq);
    g.dk = static_cast<float*>(dk);
    g.dv = static_cast<float*>(dv);
    g.status = p.status;
    g.B = B;
    g.T = T;
    g.H = H;
    g.N = N;
    g.K = K;
    g.TQ = p.TQ;
    g.qtiles = p.qtiles;
    g.scale = scale;
    g.scale_log2 = p.scale_log2;
    const int rc = H <= 16 ? launch_gather_bwd<16>(g, st) : H <= 32 ? launch_gather_bwd<32>(g, st)
                                                                     : launch_gather_bwd<64>(g, st);
    if (rc) return rc;
  }
  return WPT_OK;
}

extern "C" int wpt_f32_to_bf16(const float* x, int64_t n, void* y, void* stream) {
  if (n < 0 || (n > 0 && (!x || !y))) return fail(WPT_ERR_INVALID, "bad f32_to_bf16 arguments");
  if (n % 4 || !aligned16(x) || reinterpret_cast<uintptr_t>(y) % 8)
    return fail(WPT_ERR_INVALID, "f32_to_bf16 takes a multiple of 4 values, x 16-byte and y 8-byte aligned");
  if (n == 0) return WPT_OK;
  int sms = 148;
  current_device(&sms);
  const int64_t want = (n / 4 + 255) / 256;
  const int blocks = static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(sms) * 8));
  wpt::f32_to_bf16_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float4*>(x), n / 4, static_cast<uint2*>(y));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "f32_to_bf16_kernel launch");
  return WPT_OK;
}

extern "C" int wpt_attn_merge(const float* part_o, const float* part_lse, int splits, int64_t rows,
                              int64_t split_stride, int H, int C, const float* sink, void* out, float* lse,
                              void* stream) {
  if (C != 64 && C != 128) return fail(WPT_ERR_UNSUPPORTED, "head width %d: the kernels take 64 or 128", C);
  if (splits < 1 || rows < 0 || split_stride < rows || H < 1)
    return fail(WPT_ERR_INVALID, "bad merge shape splits=%d rows=%lld", splits, static_cast<long long>(rows));
  if (rows == 0) return WPT_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return C == 128 ? launch_merge<128>(part_o, part_lse, splits, rows, split_stride, H, sink, out, lse, s)
                  : launch_merge<64>(part_o, part_lse, splits, rows, split_stride, H, sink, out, lse, s);
}

extern "C" int wpt_attn_merge_partial(const float* part_o, const float* part_lse, int splits, int64_t rows,
                                      int64_t split_stride, int C, float* out_o, float* out_lse, void* stream) {
  if (C != 64 && C != 128) return fail(WPT_ERR_UNSUPPORTED, "head width %d: the kernels take 64 or 128", C);
  if (splits < 1 || rows < 0 || split_stride < rows)
    return fail(WPT_ERR_INVALID, "bad merge shape splits=%d rows=%lld", splits, static_cast<long long>(rows));
  if (!part_o || !part_lse || !out_o || !out_lse) return fail(WPT_ERR_INVALID, "a required pointer is NULL");
  if (rows == 0) return WPT_OK;
  wpt::SplitLayout lay;
  lay.per = splits;
  lay.stride = split_stride;
  lay.group_o = 0;
  lay.group_l = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return C == 128 ? launch_merge<128>(part_o, part_lse, splits, rows, lay, 1, nullptr, nullptr, out_lse, s, false, out_o)
                  : launch_merge<64>(part_o, part_lse, splits, rows, lay, 1, nullptr, nullptr, out_lse, s, false, out_o);
}

extern "C" int wpt_attn_merge_groups(const float* parts, int groups, int per, int64_t rows, int64_t group_floats,
                                     int H, int C, const float* sink, void* out, float* lse, void* stream) {
  if (C != 64 && C != 128) return fail(WPT_ERR_UNSUPPORTED, "head width %d: the kernels take 64 or 128", C);
  if (groups < 1 || per < 1 || rows < 0 || H < 1)
    return fail(WPT_ERR_INVALID, "bad merge shape groups=%d per=%d rows=%lld", groups, per,
                static_cast<long long>(rows));
  if (static_cast<int64_t>(groups) * per > wpt::MERGE_MAX_SPLITS * 32)
    return fail(WPT_ERR_UNSUPPORTED, "%d x %d splits: too many", groups, per);
  if (group_floats < static_cast<int64_t>(per) * rows * (C + 1))
    return fail(WPT_ERR_INVALID, "group_floats %lld < per * rows * (C + 1)", static_cast<long long>(group_floats));
  if (!parts || !out || !lse) return fail(WPT_ERR_INVALID, "a required pointer is NULL");
  if (rows == 0) return WPT_OK;
  wpt::SplitLayout lay;
  lay.per = per;
  lay.stride = rows;
  lay.group_o = group_floats;
  lay.group_l = group_floats;
  const float* part_lse = parts + static_cast<int64_t>(per) * rows * C;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int splits = groups * per;
  return C == 128 ? launch_merge<128>(parts, part_lse, splits, rows, lay, H, sink, out, lse, s)
                  : launch_merge<64>(parts, part_lse, splits, rows, lay, H, sink, out, lse, s);
}

extern "C" size_t wpt_peer_bytes(int world, int64_t rows, int C) {
  if (C != 128 || world < 1 || world > wpt::EXCH_MAX_WORLD || rows < 1 || rows > wpt::EXCH_MAX_CTAS) return 0;
  const int64_t chunk = (rows * (C + 1) + 3) / 4 * 4;
  return static_cast<size_t>(wpt::EXCH_CTRL_BYTES + 2 * world * chunk * 4);
}

extern "C" int wpt_peer_alloc(size_t bytes, void** buffer, void* handle) {
  if (bytes == 0 || !buffer || !handle) return fail(WPT_ERR_INVALID, "peer buffer: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(peer buffer)");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zeroed before any peer can write into it
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "peer buffer set-up");
  }
  std::memcpy(handle, &h, sizeof(h));
  *buffer = p;
  return WPT_OK;
}

extern "C" int wpt_peer_open(const void* handle, void** buffer) {
  if (!handle || !buffer) return fail(WPT_ERR_INVALID, "peer open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(buffer, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  return WPT_OK;
}

extern "C" int wpt_peer_close(void* buffer, int opened) {
  cudaError_t e = opened ? cudaIpcCloseMemHandle(buffer) : cudaFree(buffer);
  if (e != cudaSuccess) return cuda_fail(e, opened ? "cudaIpcCloseMemHandle" : "cudaFree(peer buffer)");
  return WPT_OK;
}

extern "C" int wpt_attn_exchange(const float* part_o, const float* part_lse, int splits, int64_t rows, int H, int C,
                                 const float* sink, void* const* peers, int world, int rank, void* out, float* lse,
                                 void* stream) {
  if (C != 128) return fail(WPT_ERR_UNSUPPORTED, "head width %d: the exchange takes 128", C);
  if (world < 1 || world > wpt::EXCH_MAX_WORLD || rank < 0 || rank >= world)
    return fail(WPT_ERR_UNSUPPORTED, "world %d rank %d: 1 to %d ranks", world, rank, wpt::EXCH_MAX_WORLD);
  if (rows < 1 || rows > wpt::EXCH_MAX_CTAS)
    return fail(WPT_ERR_UNSUPPORTED, "%lld rows: the exchange takes 1 to %d", static_cast<long long>(rows),
                wpt::EXCH_MAX_CTAS);
  if (splits < 1 || H < 1) return fail(WPT_ERR_INVALID, "bad exchange shape splits=%d H=%d", splits, H);
  if (!part_o || !part_lse || !peers || !out || !lse) return fail(WPT_ERR_INVALID, "a required pointer is NULL");
  wpt::ExchangeParams p = {};
  p.part_o = part_o;
  p.part_lse = part_lse;
  p.sink = sink;
  for (int g = 0; g < world; ++g) {
    if (!peers[g] || reinterpret_cast<uintptr_t>(peers[g]) % 256 != 0)
      return fail(WPT_ERR_INVALID, "peer buffer %d is NULL or not 256-byte aligned", g);
    p.peers[g] = static_cast<uint8_t*>(peers[g]);
  }
  p.local = p.peers[rank];
  p.out = static_cast<__nv_bfloat16*>(out);
  p.lse = lse;
  if (int rc = status_word(&p.status)) return rc;
  p.chunk = (rows * (C + 1) + 3) / 4 * 4;
  p.splits = splits;
  p.rows = static_cast<int>(rows);
  p.H = H;
  p.world = world;
  p.rank = rank;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // waits for the partials on the device
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(rows));  // one row per CTA
  cfg.blockDim = dim3(wpt::EXCH_THREADS);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaLaunchKernelEx(&cfg, wpt::exchange_kernel<128>, p);
  if (e != cudaSuccess) return cuda_fail(e, "exchange_kernel launch");
  return WPT_OK;
}

extern "C" int wpt_attn_decode(const void* q, const void* k, const void* v, int64_t k_stride_b, int64_t k_stride_n,
                               int64_t v_stride_b, int64_t v_stride_n, const int64_t* positions,
                               const int64_t* floor_rows, const int64_t* idx, int K, const float* sink, void* out,
                               float* lse, float* part_o, float* part_lse, int splits, int chunk_tiles, int B, int T,
                               int H, int C, int N, int window, float scale, void* stream) {
  if (C != 128) return fail(WPT_ERR_UNSUPPORTED, "head width %d: the key-stream kernel takes 128", C);
  if (H < 1 || H > 64) return fail(WPT_ERR_UNSUPPORTED, "%d heads: the key-stream kernel takes 1 to 64", H);
  if (B < 1 || T < 1 || N < 1) return fail(WPT_ERR_INVALID, "empty shape B=%d T=%d N=%d", B, T, N);
  if (static_cast<int64_t>(B) * T * H >= (int64_t(1) << 31)) return fail(WPT_ERR_UNSUPPORTED, "B*T*H too large");
  if (splits < 1 || chunk_tiles < 1) return fail(WPT_ERR_INVALID, "splits and chunk_tiles must be >= 1");
  if (splits > 65535) return fail(WPT_ERR_UNSUPPORTED, "%d splits: at most 65535", splits);
  // part_o and part_lse both NULL with 2..8 splits: cluster mode (the splits
  // of a group merge in shared memory; no scratch, no merge launch)
  const bool cluster = splits > 1 && part_o == nullptr && part_lse == nullptr;
  if (cluster && splits > 8) return fail(WPT_ERR_INVALID, "%d splits without scratch: at most 8", splits);
  if (splits > 1 && !cluster && (part_o == nullptr || part_lse == nullptr))
    return fail(WPT_ERR_INVALID, "splits > 1 needs both part_o and part_lse scratch (or neither, for 2 to 8)");
  if (idx != nullptr && K < 0) return fail(WPT_ERR_INVALID, "K must be >= 0");
  // out and lse both NULL with splits > 1: partials only, merged by the caller
  const bool partials_only = splits > 1 && !cluster && out == nullptr && lse == nullptr;
  if (!q || !k || !v || !positions || ((!out || !lse) && !partials_only))
    return fail(WPT_ERR_INVALID, "a required pointer is NULL");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v)) return fail(WPT_ERR_INVALID, "q, k, v must be 16-byte aligned");
  if (k_stride_n % 8 || v_stride_n % 8 || (B > 1 && (k_stride_b % 8 || v_stride_b % 8)))
    return fail(WPT_ERR_INVALID, "key/value strides must be multiples of 8 elements");
  if (!(scale > 0.f)) return fail(WPT_ERR_INVALID, "scale must be positive");
  const bool gather = idx != nullptr;
  const int cols = gather ? H : (T * H < 64 ? T * H : 64);
  const int ncol = cols <= 16 ? 16 : cols <= 32 ? 32 : 64;
  wpt::StreamParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.ksb = k_stride_b;
  p.ksn = k_stride_n;
  p.vsb = v_stride_b;
  p.vsn = v_stride_n;
  p.positions = positions;
  p.floor_rows = gather ? nullptr : floor_rows;
  p.idx = idx;
  p.K = gather ? K : 0;
  p.sink = splits > 1 && !cluster ? nullptr : sink;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.lse = lse;
  p.part_o = part_o;
  p.part_lse = part_lse;
  if (int rc = status_word(&p.status)) return rc;
  p.B = B;
  p.T = T;
  p.H = H;
  p.N = N;
  p.window = window > 0 ? window : 0;
  p.TQ = gather ? 1 : ncol / H;
  p.groups_per_row = (T + p.TQ - 1) / p.TQ;
  p.splits = splits;
  p.chunk_tiles = chunk_tiles;
  p.cluster = cluster ? splits : 0;
  p.scale_log2 = scale * wpt::LOG2E;
  const int64_t groups = static_cast<int64_t>(B) * p.groups_per_row;
  if (groups >= (int64_t(1) << 31)) return fail(WPT_ERR_UNSUPPORTED, "too many query groups");
  // range mode loads whole tiles by TMA; gather mode loads its window's
  // tiles by TMA when the tables allow tensor maps, else copies every row
  CUtensorMap tk, tv;
  memset(&tk, 0, sizeof(tk));
  memset(&tv, 0, sizeof(tv));
  const auto mappable = [&](const void* t, int64_t sb, int64_t sn) {
    return aligned16(t) && sn % 8 == 0 && (B == 1 || sb % 8 == 0) && sn >= C;
  };
  p.window_tma = 0;
  if (!gather || (mappable(k, k_stride_b, k_stride_n) && mappable(v, v_stride_b, v_stride_n) && window > 0)) {
    if (int rc = table_map(&tk, k, k_stride_b, k_stride_n, B, N, C)) return rc;
    if (int rc = table_map(&tv, v, v_stride_b, v_stride_n, B, N, C)) return rc;
    p.window_tma = gather ? 1 : 0;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rc = gather ? launch_stream_g<true>(tk, tv, p, ncol, static_cast<int>(groups), s)
                        : launch_stream_g<false>(tk, tv, p, ncol, static_cast<int>(groups), s);
  if (rc) return rc;
  if (splits > 1 && !partials_only && !cluster) {
    const int64_t rows = static_cast<int64_t>(B) * T * H;
    return launch_merge<128>(part_o, part_lse, splits, rows, rows, H, sink, out, lse, s, true);
  }
  return WPT_OK;
}

extern "C" int wpt_attn_topk(const void* q, const void* k, int64_t k_stride_b, int64_t k_stride_n,
                             const int64_t* positions, const float* lse, float* scores, int64_t ld_scores,
                             int64_t* chosen, int K, int B, int T, int H, int C, int N, int window, float scale,
                             void* stream) {
  if (C != 128) return fail(WPT_ERR_UNSUPPORTED, "head width %d: the selection kernel takes 128", C);
  if (H < 1 || H > 128) return fail(WPT_ERR_UNSUPPORTED, "%d heads: the selection kernel takes 1 to 128", H);
  if (B < 1 || T < 1 || N < 1 || K < 0) return fail(WPT_ERR_INVALID, "bad shape B=%d T=%d N=%d K=%d", B, T, N, K);
  if (K == 0) return WPT_OK;
  if (ld_scores < N) return fail(WPT_ERR_INVALID, "ld_scores %lld < N %d", static_cast<long long>(ld_scores), N);
  if (!q || !k || !positions || !lse || !scores || !chosen) return fail(WPT_ERR_INVALID, "a required pointer is NULL");
  if (!aligned16(q)) return fail(WPT_ERR_INVALID, "q must be 16-byte aligned");
  if (static_cast<int64_t>(B) * T * H >= (int64_t(1) << 31)) return fail(WPT_ERR_UNSUPPORTED, "B*T*H too large");
  const int cols = T * H < 256 ? T * H : 256;
  const int ncol = cols <= 16 ? 16 : cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : 256;
  wpt::ScoreParams p;
  p.positions = positions;
  p.lse = lse;
  p.scores = scores;
  p.ld = ld_scores;
  if (int rc = status_word(&p.status)) return rc;
  p.B = B;
  p.T = T;
  p.H = H;
  p.N = N;
  p.window = window;
  p.TQ = ncol / H;
  if (p.TQ < 1) return fail(WPT_ERR_UNSUPPORTED, "%d heads exceed the selection kernel's columns", H);
  p.groups_per_row = (T + p.TQ - 1) / p.TQ;
  p.scale = scale;
  const int64_t groups = static_cast<int64_t>(B) * p.groups_per_row;
  // one query per group (decode) and few groups: the groups' live key tiles
  // split evenly over one CTA per SM, whatever the rows' lengths
  p.balanced = T == 1 && p.TQ == 1 && groups <= wpt::SCORE_BAL_GROUPS ? 1 : 0;
  const int tiles = (N + 127) / 128;
  int64_t chunk = (static_cast<int64_t>(tiles) * groups + 4 * 148 - 1) / (4 * 148);
  if (chunk < 4) chunk = 4;
  if (chunk > tiles) chunk = tiles;
  p.chunk_tiles = static_cast<int>(chunk);
  const int splits = (tiles + p.chunk_tiles - 1) / p.chunk_tiles;
  if (groups >= (int64_t(1) << 31) || splits > 65535) return fail(WPT_ERR_UNSUPPORTED, "selection grid too large");
  CUtensorMap tq, tk;
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(B) * T * H};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(C) * 2};
    cuuint32_t box[2] = {64, static_cast<cuuint32_t>(ncol)};
    if (int rc = tensor_map(&tq, q, 2, dims, strides, box)) return rc;
  }
  if (int rc = table_map(&tk, k, k_stride_b, k_stride_n, B, N, C)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc;
  switch (ncol) {
    case 16: rc = launch_score<16>(tq, tk, p, static_cast<int>(groups), splits, s); break;
    case 32: rc = launch_score<32>(tq, tk, p, static_cast<int>(groups), splits, s); break;
    case 64: rc = launch_score<64>(tq, tk, p, static_cast<int>(groups), splits, s); break;
    case 128: rc = launch_score<128>(tq, tk, p, static_cast<int>(groups), splits, s); break;
    default: rc = launch_score<256>(tq, tk, p, static_cast<int>(groups), splits, s); break;
  }
  if (rc) return rc;
  const int cap = N < 47104 ? N : 47104;  // keys cached in shared memory (the rest of it: bins, candidates)
  const int smem = (cap + 1 + wpt::SELECT_BINS + 2 * wpt::SELECT_CAND + 64) * 4;
  int sms = 148;
  current_device(&sms);
  const int64_t queries = static_cast<int64_t>(B) * T;
  // fewer queries than SMs: each query's candidates in two slices, a 2-CTA
  // cluster per query (WPT_B200_TOPK_PAIR=0 keeps one CTA)
  static const int pair_env = [] {
    const char* env = getenv("WPT_B200_TOPK_PAIR");
    return env ? atoi(env) : 1;
  }();
  const bool pair = pair_env != 0 && queries < sms;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // waits for the scores on the device
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pair ? 2 : 1;
  cfg.gridDim = dim3(static_cast<unsigned>(pair ? 2 * queries : queries));
  cfg.blockDim = dim3(wpt::TOPK_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaError_t e;
  if (pair) {
    if (int rc2 = allow_smem(wpt::topk_kernel<2>, smem)) return rc2;
    e = cudaLaunchKernelEx(&cfg, wpt::topk_kernel<2>, scores, ld_scores, positions, chosen, T, N, K, window, cap);
  } else {
    if (int rc2 = allow_smem(wpt::topk_kernel<1>, smem)) return rc2;
    e = cudaLaunchKernelEx(&cfg, wpt::topk_kernel<1>, scores, ld_scores, positions, chosen, T, N, K, window, cap);
  }
  if (e != cudaSuccess) return cuda_fail(e, "topk_kernel launch");
  return WPT_OK;
}

extern "C" int wpt_tree_bits(const int64_t* parents, int64_t parents_stride_b, int B, int n, uint64_t* bits,
                             const int64_t* base, int64_t* positions, void* stream) {
  if (B < 1 || n < 1) return fail(WPT_ERR_INVALID, "empty tree batch B=%d n=%d", B, n);
  if (n > 64) return fail(WPT_ERR_UNSUPPORTED, "a tree of %d nodes: the kernels take up to 64", n);
  if (!parents || !bits || (positions && !base)) return fail(WPT_ERR_INVALID, "a required pointer is NULL");
  if (parents_stride_b != 0 && parents_stride_b < n)
    return fail(WPT_ERR_INVALID, "parents_stride_b must be 0 (one tree for every row) or at least n");
  const int64_t total = static_cast<int64_t>(B) * n;
  const int64_t blocks = (total + 255) / 256;
  if (blocks >= (int64_t(1) << 31)) return fail(WPT_ERR_UNSUPPORTED, "too many tree rows");
  wpt::tree_bits_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      parents, parents_stride_b, B, n, bits, base, positions);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "tree_bits_kernel launch");
  return WPT_OK;
}

extern "C" int wpt_cache_append(const void* src, int64_t src_stride_b, int64_t src_stride_n, void* dst,
                                int64_t dst_stride_b, int64_t dst_stride_n, const int64_t* first,
                                const int64_t* counts, int B, int n, int row_bytes, int64_t capacity, void* stream) {
  if (B < 0 || n < 0 || row_bytes < 0 || capacity < 0) return fail(WPT_ERR_INVALID, "bad cache_append shape");
  if (B == 0 || n == 0 || row_bytes == 0) return WPT_OK;
  if (!src || !dst || !first || !counts) return fail(WPT_ERR_INVALID, "a required pointer is NULL");
  if (row_bytes % 16 || src_stride_b % 16 || src_stride_n % 16 || dst_stride_b % 16 || dst_stride_n % 16 ||
      !aligned16(src) || !aligned16(dst))
    return fail(WPT_ERR_INVALID, "cache_append copies 16-byte units: rows, strides and bases must be 16-byte multiples");
  unsigned* status = nullptr;
  if (int rc = status_word(&status)) return rc;
  const int64_t warps = static_cast<int64_t>(B) * n;
  const int64_t blocks = (warps + 7) / 8;
  if (blocks >= (int64_t(1) << 31)) return fail(WPT_ERR_UNSUPPORTED, "too many rows to append");
  wpt::cache_append_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src), src_stride_b, src_stride_n, static_cast<uint8_t*>(dst), dst_stride_b,
      dst_stride_n, first, counts, B, n, row_bytes, capacity, status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "cache_append_kernel launch");
  return WPT_OK;
}

extern "C" int wpt_temperature_scale(const float* x, int64_t n, float temperature, float* out, void* stream) {
  if (n < 0 || (n > 0 && (!x || !out))) return fail(WPT_ERR_INVALID, "bad temperature_scale arguments");
  if (!(temperature > 0.f)) return fail(WPT_ERR_INVALID, "temperature must be positive");
  if (n == 0) return WPT_OK;
  int sms = 148;
  current_device(&sms);
  const int64_t want = (n + 255) / 256;
  const int blocks = static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(sms) * 8));
  wpt::temperature_scale_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, n, temperature, out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "temperature_scale_kernel launch");
  return WPT_OK;
}

extern "C" size_t wpt_accept_scratch_bytes(int R, int n, int V) {
  if (R < 0 || n < 0 || V < 1) return 0;
  return wpt::accept_scratch(R, n, V).bytes;
}

namespace {
template <int N>
int launch_head(const CUtensorMap& tw, const CUtensorMap& th, const wpt::HeadParams& p, cudaStream_t stream) {
  using L = wpt::HeadLayout<N>;
  static_assert(L::BYTES <= 232448, "head kernel shared memory exceeds 227 KB");
  auto kernel = wpt::head_kernel<N>;
  if (int rc = allow_smem(kernel, L::BYTES)) return rc;
  int sms = 148;
  current_device(&sms);
  const int grid = p.tiles < sms ? p.tiles : sms;  // persistent: one CTA per SM walks the vocabulary tiles
  kernel<<<grid, wpt::HEAD_THREADS, L::BYTES, stream>>>(tw, th, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "head_kernel launch");
  return WPT_OK;
}
}  // namespace

extern "C" int wpt_head_scores(const void* h, int64_t h_stride, const void* w, int64_t w_stride, int R, int D,
                               int V, int round_bf16, float* scores, void* stream) {
  if (R < 1 || D < 1 || V < 1) return fail(WPT_ERR_INVALID, "empty shape R=%d D=%d V=%d", R, D, V);
  if (D % 64 != 0) return fail(WPT_ERR_UNSUPPORTED, "model width %d: the head kernel takes multiples of 64", D);
  if (!h || !w || !scores) return fail(WPT_ERR_INVALID, "a required pointer is NULL");
  if (!aligned16(h) || !aligned16(w)) return fail(WPT_ERR_INVALID, "h and the head weight must be 16-byte aligned");
  if (h_stride < D || w_stride < D || h_stride % 8 || w_stride % 8)
    return fail(WPT_ERR_INVALID, "row strides must be at least D and multiples of 8 elements");
  if (static_cast<int64_t>(R) * V >= (int64_t(1) << 40)) return fail(WPT_ERR_UNSUPPORTED, "R*V too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int tiles = (V + 127) / 128;
  CUtensorMap tw;
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(V)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(w_stride) * 2};
    cuuint32_t box[2] = {64, 128};
    if (int rc = tensor_map(&tw, w, 2, dims, strides, box)) return rc;
  }
  for (int r0 = 0; r0 < R; r0 += 128) {  // up to 128 rows of h per launch (the MMA's N)
    const int rows = R - r0 < 128 ? R - r0 : 128;
    const int n = rows <= 32 ? 32 : rows <= 64 ? 64 : 128;
    const void* hb = static_cast<const __nv_bfloat16*>(h) + static_cast<int64_t>(r0) * h_stride;
    CUtensorMap th;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(h_stride) * 2};
    cuuint32_t box[2] = {64, static_cast<cuuint32_t>(n)};
    if (int rc = tensor_map(&th, hb, 2, dims, strides, box)) return rc;
    wpt::HeadParams p;
    p.scores = scores + static_cast<int64_t>(r0) * V;
    if (int rc = status_word(&p.status)) return rc;
    p.R = rows;
    p.V = V;
    p.D = D;
    p.tiles = tiles;
    p.round_bf16 = round_bf16 ? 1 : 0;
    const int rc = n == 32 ? launch_head<32>(tw, th, p, s) : n == 64 ? launch_head<64>(tw, th, p, s)
                                                                     : launch_head<128>(tw, th, p, s);
    if (rc) return rc;
  }
  return WPT_OK;
}

extern "C" int wpt_accept(const float* scores, const int64_t* drafted, const float* q, const float* uniforms,
                          const float* resample, const int64_t* lengths, void* scratch, int64_t* tokens,
                          int64_t* accepted, int R, int n, int V, float temperature, int top_k, void* stream) {
  if (R < 0 || n < 0 || V < 1) return fail(WPT_ERR_INVALID, "bad accept shape R=%d n=%d V=%d", R, n, V);
  if (R == 0) return WPT_OK;
  if (R > 65535 || n + 1 > 65535) return fail(WPT_ERR_UNSUPPORTED, "accept grid too large (R=%d, n=%d)", R, n);
  if (!(temperature > 0.f)) return fail(WPT_ERR_INVALID, "temperature must be positive");
  if (!scores || !scratch || !tokens || !accepted || !resample || (n > 0 && (!drafted || !q || !uniforms)))
    return fail(WPT_ERR_INVALID, "a required pointer is NULL");
  if (reinterpret_cast<uintptr_t>(scratch) % 16 != 0) return fail(WPT_ERR_INVALID, "accept scratch not 16-byte aligned");
  const wpt::AcceptScratch layout = wpt::accept_scratch(R, n, V);
  char* base = static_cast<char*>(scratch);
  wpt::AcceptParams p;
  p.scores = scores;
  p.drafted = drafted;
  p.q = q;
  p.uniforms = uniforms;
  p.resample = resample;
  p.lengths = lengths;
  p.part = reinterpret_cast<float2*>(base + layout.part);
  p.pos_stat = reinterpret_cast<float2*>(base + layout.pos_stat);
  p.thr = reinterpret_cast<float*>(base + layout.thr);
  p.keep = reinterpret_cast<int*>(base + layout.keep);
  p.chunk_sum = reinterpret_cast<double*>(base + layout.chunk_sum);
  p.pos_count = reinterpret_cast<unsigned*>(base + layout.pos_count);
  p.count = reinterpret_cast<unsigned*>(base + layout.count);
  p.ticket = reinterpret_cast<unsigned long long*>(base + layout.ticket);
  p.tokens = tokens;
  p.accepted = accepted;
  p.R = R;
  p.n = n;
  p.V = V;
  p.top_k = top_k;
  p.S = (V + wpt::STAT_SEG - 1) / wpt::STAT_SEG;
  p.chunks = (V + wpt::DRAW_CHUNK - 1) / wpt::DRAW_CHUNK;
  p.temperature = temperature;
  const int slices = (p.chunks + wpt::DRAW_CPS - 1) / wpt::DRAW_CPS;
  if (slices > 65535) return fail(WPT_ERR_UNSUPPORTED, "vocabulary of %d entries is too large", V);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the arrival counters (positions', rows') and the unit ticket start at zero
  cudaError_t e = cudaMemsetAsync(base + layout.pos_count, 0, layout.bytes - layout.pos_count, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(accept counters)");
  if (top_k > 1 && top_k < V) {
    wpt::accept_topk_stats_kernel<<<dim3(n + 1, R), wpt::ACCEPT_THREADS, 0, s>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "accept_topk_stats_kernel launch");
  } else {
    // a grid the SMs hold at once: its warps take the units in turn
    const bool greedy = top_k == 1 && V > 1;
    const int variant = (greedy ? 2 : 0) + (temperature == 1.f ? 1 : 0);
    void (*const kernels[4])(const wpt::AcceptParams) = {
        wpt::accept_stats_kernel<false, false>, wpt::accept_stats_kernel<false, true>,
        wpt::accept_stats_kernel<true, false>, wpt::accept_stats_kernel<true, true>};
    auto kernel = kernels[variant];
    static int resident[4][64] = {};
    int sms = 148;
    const int dev = current_device(&sms);
    if (resident[variant][dev] == 0) {
      int per_sm = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, wpt::STAT_THREADS, 0);
      if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
      resident[variant][dev] = per_sm > 0 ? per_sm : 1;
    }
    const int64_t units = static_cast<int64_t>(R) * (n + 1) * p.S;
    const int64_t want = (units + wpt::STAT_THREADS / 32 - 1) / (wpt::STAT_THREADS / 32);
    const int blocks = static_cast<int>(
        std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(sms) * resident[variant][dev])));
    kernel<<<blocks, wpt::STAT_THREADS, 0, s>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "accept_stats_kernel launch");
  }
  // the draw launches while the statistics finish (programmatic dependent
  // launch) and waits for them on the device
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(R, slices);
  cfg.blockDim = dim3(wpt::DRAW_THREADS);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, wpt::accept_draw_kernel, p);
  if (e != cudaSuccess) return cuda_fail(e, "accept_draw_kernel launch");
  return WPT_OK;
}

// ---------------------------------------------------------------- no-alloc
// Scratch of wpt_attn_decode_noalloc: the per-split partial outputs and
// log-sum-exps live in this file-scope device array instead of buffers the
// caller allocates. Every GPU that loads the library holds these 8 MiB
// until the process exits. In host code the array's name is only a
// host-side stand-in: its device address comes from cudaGetSymbolAddress,
// once per device, with that device current.
constexpr size_t WPT_NOALLOC_SCRATCH_FLOATS = size_t(1) << 21;  // 8 MiB of fp32
static __device__ __align__(256) float g_noalloc_scratch[WPT_NOALLOC_SCRATCH_FLOATS];

namespace {

int noalloc_scratch(float** out) {
  static float* cached[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(WPT_ERR_INVALID, "device %d out of range", dev);
  std::lock_guard<std::mutex> guard(g_symbol_lock);
  if (cached[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    cached[dev] = static_cast<float*>(p);
  }
  *out = cached[dev];
  return WPT_OK;
}

}  // namespace

extern "C" int wpt_attn_decode_noalloc(const void* q, const void* k, const void* v, int64_t k_stride_b,
                                       int64_t k_stride_n, int64_t v_stride_b, int64_t v_stride_n,
                                       const int64_t* positions, const int64_t* floor_rows, const int64_t* idx,
                                       int K, const float* sink, void* out, float* lse, int splits, int chunk_tiles,
                                       int B, int T, int H, int C, int N, int window, float scale, void* stream) {
  // The partials live in the library's private array, where the caller
  // cannot read them: the partials-only mode of wpt_attn_decode
  // (out == lse == NULL) would compute nothing the caller can see.
  if (out == nullptr || lse == nullptr)
    return fail(WPT_ERR_INVALID, "no-alloc decode: out and lse are required (its partials are not readable)");
  if (C != 128) return fail(WPT_ERR_UNSUPPORTED, "head width %d: the key-stream kernel takes 128", C);
  if (H < 1 || H > 64) return fail(WPT_ERR_UNSUPPORTED, "%d heads: the key-stream kernel takes 1 to 64", H);
  if (B < 1 || T < 1) return fail(WPT_ERR_INVALID, "empty shape B=%d T=%d", B, T);
  if (splits < 1) return fail(WPT_ERR_INVALID, "splits must be >= 1");
  if (splits > 65535) return fail(WPT_ERR_UNSUPPORTED, "%d splits: at most 65535", splits);
  const int64_t rows = static_cast<int64_t>(B) * T * H;
  if (rows >= (int64_t(1) << 31)) return fail(WPT_ERR_UNSUPPORTED, "B*T*H = %lld rows is too many",
                                              static_cast<long long>(rows));
  float* part_o = nullptr;
  float* part_lse = nullptr;
  if (splits > 1) {
    // splits < 2^16 and rows < 2^31, so the product fits in 64 bits
    const int64_t need = static_cast<int64_t>(splits) * rows * (C + 1);
    if (need > static_cast<int64_t>(WPT_NOALLOC_SCRATCH_FLOATS))
      return fail(WPT_ERR_UNSUPPORTED,
                  "no-alloc decode: %d splits x %lld rows x (%d + 1) floats = %lld floats exceed the %lld-float "
                  "(8 MiB) static scratch; use fewer splits or rows, or wpt_attn_decode with caller buffers",
                  splits, static_cast<long long>(rows), C, static_cast<long long>(need),
                  static_cast<long long>(WPT_NOALLOC_SCRATCH_FLOATS));
    float* scratch = nullptr;
    if (int rc = noalloc_scratch(&scratch)) return rc;
    part_o = scratch;                                   // (splits, rows, C), 256-byte aligned
    part_lse = scratch + static_cast<int64_t>(splits) * rows * C;  // (splits, rows)
  }
  return wpt_attn_decode(q, k, v, k_stride_b, k_stride_n, v_stride_b, v_stride_n, positions, floor_rows, idx, K, sink,
                         out, lse, part_o, part_lse, splits, chunk_tiles, B, T, H, C, N, window, scale, stream);
}
