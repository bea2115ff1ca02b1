/*
 * wpt_attn.h: the C ABI of the B200 (sm_100a) attention library
 * libwpt_b200.so. Plain pointers, sizes and a CUDA stream handle; no torch
 * types. Every entry point that computes only enqueues work on `stream` (no
 * host synchronisation, no allocation: buffers, including scratch, come from
 * the caller; the long row's one-time exchange set-up, wpt_peer_alloc and
 * wpt_peer_open, is the exception) and returns WPT_OK or an error code whose
 * text wpt_last_error() gives.
 *
 * These replace the kernel-form contract of the reference (paths relative
 * to the reference repository, packages/wpt-model/src/wpt_model/):
 *   pytorch_kernels.py:18-26   the contract: q (B, T, H, c), k and v (B, N, c)
 *                              in one dtype, positions (B, T) int64, sink (H,)
 *                              fp32, indices (B, T, K) int64 with -1 for none
 *   kernels.py:161-184         exact_attention / sparse_attention dispatch
 *   attention.py:85-107        window_attention
 *   packages/wpt-inference/src/wpt_inference/__init__.py:173-179,210-222
 *                              the speculative-decoding acceptance step
 *
 * Conventions shared by the attention entry points:
 *   q, out     bf16, contiguous (B, T, H, C); C is 64 or 128, H <= 128.
 *   k, v       bf16 tables (B, N, C) with the last dim contiguous and any
 *              row / batch strides (in elements, multiples of 8), e.g. the
 *              two halves of one (B, N, 2C) entries table.
 *   positions  int64 (B, T): each query's own row. A query reads rows up to
 *              min(position, N - 1) (pytorch_kernels.py:18-26: a padding query
 *              past the table reads up to its last row).
 *   lse        fp32 (B, T, H): natural-log softmax denominators, the sink's
 *              term included when a sink is given.
 *   scale      the softmax scale (c ** -0.5 in WPT).
 *   stream     a cudaStream_t (e.g. torch.cuda.current_stream().cuda_stream).
 */
#ifndef WPT_ATTN_H_
#define WPT_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  WPT_OK = 0,
  WPT_ERR_INVALID = 1,      /* an argument breaks the contract */
  WPT_ERR_UNSUPPORTED = 2,  /* a shape this library does not compute (e.g. C not 64 or 128) */
  WPT_ERR_CUDA = 3          /* a CUDA call failed */
};

/* Text of the last error on this host thread. */
const char* wpt_last_error(void);

/* The device-side status word of the current device (bit 0: an mbarrier
 * wait ran out of time, bit 1: a kernel met a shape it does not handle);
 * synchronises the device. reset != 0 clears it after reading. */
int wpt_status(unsigned* status, int reset);

/*
 * Attention of many queries per batch row over a contiguous range of rows,
 * on the tensor cores (tcgen05, TMEM accumulators, TMA-fed tiles).
 * Replaces exact_attention's forward (pytorch_kernels.py:98-121; the
 * Triton form's _exact_forward_kernel, triton_kernels.py:300-326) and the
 * window/sink attention (pytorch_kernels.py:171-187 over the window rows
 * :149-153; attention.py:85-107), and computes tree-masked verification.
 *   window      > 0: a query at position p reads rows p - window + 1 .. p
 *   floor_rows  int64 (B, T) or NULL: the lowest row each query may read
 *   tree_bits   uint64 (B, T) or NULL: rows tree_base[b] + i, i < 64, are
 *               visible to query t only when bit i of tree_bits[b, t] is set
 *   tree_base   int64 (B,) or NULL (required with tree_bits)
 *   sink        fp32 (H,) or NULL: one logit per head added to the denominator
 *   splits      > 1 splits each CTA's rows; part_o (splits, B*T*H, C) fp32
 *               and part_lse (splits, B*T*H) fp32 are then caller scratch.
 *               splits == 2 with part_o == part_lse == NULL: cluster mode,
 *               for shapes of at most one work item (pair of 128-row query
 *               tiles and split) per SM: a pair's two splits run as one
 *               2-CTA cluster and combine in shared memory (no scratch, no
 *               merge launch); more items than SMs return WPT_ERR_INVALID
 */
int wpt_attn_prefill(const void* q, const void* k, const void* v, int64_t k_stride_b, int64_t k_stride_n,
                     int64_t v_stride_b, int64_t v_stride_n, const int64_t* positions, const int64_t* floor_rows,
                     const uint64_t* tree_bits, const int64_t* tree_base, const float* sink, void* out, float* lse,
                     float* part_o, float* part_lse, int splits, int B, int T, int H, int C, int N, int window,
                     float scale, void* stream);

/*
 * Attention of few queries per batch row (decode, short extends) or of
 * gathered rows (sparse), on the tensor cores with the keys as the MMA's M
 * (S^T = K Q^T), split over CTAs along the keys. Replaces exact_attention's
 * decode use (pytorch_kernels.py:98-121 at T = 1; the Triton form's (1, B)
 * grid, triton_kernels.py:216) and sparse_attention
 * (pytorch_kernels.py:171-187,213-217; triton_kernels.py:681-716).
 *   idx == NULL  range mode: as wpt_attn_prefill (positions, window,
 *                floor_rows); up to 64 / H queries share a CTA
 *   idx != NULL  gather mode: idx int64 (B, T, K), -1 for none; each query
 *                reads its rows idx[b, t, :] and then its last `window`
 *                rows (rows < 0 or >= N are skipped), with the sink
 *   splits, chunk_tiles  each query group's rows are cut into chunks of
 *                chunk_tiles * 128 and chunk s goes to split s; rows past
 *                splits * chunk_tiles * 128 are not read, so splits must
 *                cover the longest row. splits > 1 needs part_o
 *                (splits, B*T*H, C) and part_lse (splits, B*T*H) fp32 scratch,
 *                or both NULL with 2 to 8 splits: cluster mode, where each
 *                group's splits run as one thread-block cluster and combine
 *                in shared memory (no scratch, no second kernel). Cluster
 *                mode suits grids of one wave (groups * splits at most the
 *                SM count): a cluster holds its SMs until its last split ends.
 *   out == lse == NULL with splits > 1: the call stops at the partials
 *                (each split's output normalised by its own sum, and the
 *                natural log of that sum; no sink), for a caller that merges
 *                them with other partials (wpt_attn_merge), e.g. those of
 *                the other GPUs holding the rest of a long row.
 *   C must be 128 and H at most 64.
 */
int wpt_attn_decode(const void* q, const void* k, const void* v, int64_t k_stride_b, int64_t k_stride_n,
                    int64_t v_stride_b, int64_t v_stride_n, const int64_t* positions, const int64_t* floor_rows,
                    const int64_t* idx, int K, const float* sink, void* out, float* lse, float* part_o,
                    float* part_lse, int splits, int chunk_tiles, int B, int T, int H, int C, int N, int window,
                    float scale, void* stream);

/*
 * Exact attention's choice of rows (HySparse2's oracle selection,
 * pytorch_kernels.py:112-117; the Triton form's _exact_choice_kernel,
 * triton_kernels.py:393-508): for each query at position p, the K rows
 * among 0 .. min(p - window, N - 1) with the largest
 * score(n) = max_h (q_h . k_n * scale - lse_h), written to chosen (B, T, K)
 * int64: the rows above the K-th score first, then rows equal to it by
 * row index; every candidate in row order, then -1, when a query has K or
 * fewer. lse (B, T, H) fp32 is the forward pass's. scores is caller scratch
 * of B * T * ld_scores fp32 (ld_scores >= N). C must be 128, H at most 128.
 * K = chosen_columns(top_k, window, N) (pytorch_kernels.py:73-77).
 */
int wpt_attn_topk(const void* q, const void* k, int64_t k_stride_b, int64_t k_stride_n, const int64_t* positions,
                  const float* lse, float* scores, int64_t ld_scores, int64_t* chosen, int K, int B, int T, int H,
                  int C, int N, int window, float scale, void* stream);

/*
 * wpt_attn_decode without caller scratch: the same computation and
 * arguments, but the split partials go to a static 8 MiB device array the
 * library holds on every GPU that loads it, so the call allocates nothing.
 * No counterpart in the reference. It serves callers that cannot allocate
 * device memory per call: a host behind an FFI (Go, Java, Rust) with no
 * caching allocator, where a cudaMalloc and cudaFree per step would
 * synchronise the device, or a serving process that must not grow its
 * footprint mid-run.
 * Limit: splits * B * T * H * (C + 1) floats must fit in 2^21 (8 MiB);
 * larger calls return WPT_ERR_UNSUPPORTED and launch nothing. out and lse
 * are required (WPT_ERR_INVALID when NULL): the partials-only mode of
 * wpt_attn_decode would leave its results in the private array, where the
 * caller cannot read them. The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress); make that first call before any
 * stream capture. That address (like the status word's) is cached for the
 * life of the process: do not use the library across a cudaDeviceReset.
 * Every call shares the array: calls that overlap on the GPU (other
 * streams, other threads) race on it, so serialise them. Nothing in the
 * array needs to start at zero: each call writes every partial its merge
 * reads.
 */
int wpt_attn_decode_noalloc(const void* q, const void* k, const void* v, int64_t k_stride_b, int64_t k_stride_n,
                            int64_t v_stride_b, int64_t v_stride_n, const int64_t* positions,
                            const int64_t* floor_rows, const int64_t* idx, int K, const float* sink, void* out,
                            float* lse, int splits, int chunk_tiles, int B, int T, int H, int C, int N, int window,
                            float scale, void* stream);

/*
 * Merge of split-KV partial results (o normalised per split, fp32; lse per
 * split, natural log, -inf for none) into out (bf16) and lse, adding the
 * sink. part_o (splits, rows, C) at split stride split_stride rows;
 * part_lse (splits, rows). rows = B*T*H, head = row % H. Used by the
 * split-KV paths and by the multi-GPU long-sequence decode (merges the
 * GPUs' partials after an NCCL all-gather). No reference counterpart
 * beyond the log-sum-exp algebra of pytorch_kernels.py:183-184.
 */
int wpt_attn_merge(const float* part_o, const float* part_lse, int splits, int64_t rows, int64_t split_stride,
                   int H, int C, const float* sink, void* out, float* lse, void* stream);

/*
 * Gradients of the attention above (exact, window/sink, and sparse with
 * chosen rows), on the tensor cores, from the forward pass's out (bf16) and
 * lse. Replaces the backward passes of the reference's forms: the PyTorch
 * form's _Exact.backward and _Sparse.backward (pytorch_kernels.py:123-139,
 * 189-210) and the Triton form's _exact_backward_kernel and sparse backward
 * kernels (triton_kernels.py:546-571, 719-908).
 *   positions, floor_rows, window  the rows each query read, as in
 *                wpt_attn_prefill (range part)
 *   idx, K       idx (B, T, K) int64 chosen rows (-1 for none), read on top
 *                of the range part (sparse_attention's rows: chosen, then the
 *                last `window`); K = 0 / idx NULL for exact or window attention
 *   sink         fp32 (H,) or NULL; d_sink fp32 (H,) or NULL receives its
 *                gradient, -sum exp(sink - lse) delta (deterministic order)
 *   d_out        bf16 (B, T, H, C) contiguous
 *   dq           (B, T, H, C); dk, dv (B, N, C), contiguous; bf16, or fp32 when
 *                f32_grads != 0 (required when K > 0: chosen rows are added
 *                by fp32 atomics; wpt_f32_to_bf16 converts)
 *   scratch      wpt_attn_backward_scratch_bytes(B, T, H, C, N) bytes, 16-byte aligned
 * C must be 128, H at most 128 (64 with chosen rows).
 */
int wpt_attn_backward(const void* q, const void* k, const void* v, int64_t k_stride_b, int64_t k_stride_n,
                      int64_t v_stride_b, int64_t v_stride_n, const int64_t* positions, const int64_t* floor_rows,
                      const int64_t* idx, int K, const float* sink, const void* out, const float* lse,
                      const void* d_out, void* dq, void* dk, void* dv, float* d_sink, void* scratch, int f32_grads,
                      int B, int T, int H, int C, int N, int window, float scale, void* stream);

/*
 * Failure-detection test hook (no counterpart in the reference; tests only).
 * From the next wpt_attn_backward call on, the query-tile kernel's loader
 * does not issue the copy of key tile `skip_key_tile` of each of its CTAs
 * (-1: off), and that kernel's mbarrier waits give up after wait_ns
 * nanoseconds (0: the default, 2 s). A wait that gives up sets bit 0 of the
 * status word (wpt_status), every role of the CTA stops, the loader lets
 * the copies it did issue land, TMEM is freed and the kernel returns: the
 * context stays usable, and the gradients of that call are not written.
 * Nothing is ever in flight for the skipped tile, so nothing lands late.
 */
int wpt_debug_backward_fault(int skip_key_tile, unsigned long long wait_ns);

/* Bytes of scratch wpt_attn_backward needs (0 for a shape it does not take). */
size_t wpt_attn_backward_scratch_bytes(int B, int T, int H, int C, int N);

/* y[i] = bf16(x[i]) (round to nearest even) for n fp32 values, n a multiple
 * of 4, x 16-byte and y 8-byte aligned. */
int wpt_f32_to_bf16(const float* x, int64_t n, void* y, void* stream);

/*
 * The same merge without a sink, its result kept as a partial: out_o
 * (rows, C) fp32, the splits' output normalised by their common sum, and
 * out_lse (rows,) its natural log. Several GPUs that each hold a share of a
 * long row's keys merge their own splits this way, so that one small
 * partial per GPU is all they exchange.
 */
int wpt_attn_merge_partial(const float* part_o, const float* part_lse, int splits, int64_t rows, int64_t split_stride,
                           int C, float* out_o, float* out_lse, void* stream);

/*
 * The same merge over partials gathered from several places (the GPUs that
 * each hold a share of a long row's keys): `groups` chunks of group_floats
 * floats side by side at `parts`, chunk g holding `per` splits' output
 * partials (per, rows, C) fp32 followed by their log-sums (per, rows) fp32
 * (group_floats >= per * rows * (C + 1); pad it to keep chunks 16-byte
 * aligned). One wpt_attn_decode call in partials-only mode writes such a
 * chunk (part_o = the chunk, part_lse = the chunk + per * rows * C), so an
 * in-place all-gather of the chunks is the only exchange a long row needs.
 * No reference counterpart (the reference decodes on one GPU).
 */
int wpt_attn_merge_groups(const float* parts, int groups, int per, int64_t rows, int64_t group_floats, int H, int C,
                          const float* sink, void* out, float* lse, void* stream);

/*
 * The long row's exchange without a collective library (no reference
 * counterpart: the reference decodes on one GPU). Each rank of a long row
 * whose keys are split over `world` GPUs (one process per GPU, never two
 * ranks on one GPU: the ranks' kernels wait for one another) sets up once:
 *   wpt_peer_bytes(world, rows, C)   bytes of its exchange buffer (0: the
 *                                    shape is not taken: C 128, world
 *                                    1..8, rows 1..4096)
 *   wpt_peer_alloc(bytes, &buf, h)   cudaMalloc + zero-fill + synchronise;
 *                                    h receives its 64-byte CUDA IPC handle
 *   (the caller exchanges the handles, e.g. over its process group)
 *   wpt_peer_open(h_peer, &ptr)      maps a peer's buffer into this process
 *   (then a barrier over the ranks: no rank may write into a buffer before
 *   its owner has zeroed it)
 *   wpt_peer_close(ptr, opened)      unmaps (opened = 1) or frees (0)
 * Per call, after this rank's split partials (wpt_attn_decode in
 * partials-only mode over its shard), wpt_attn_exchange launches one kernel
 * that merges them, stores the result into every rank's buffer through the
 * mappings (NVLink), signals each rank, waits (bounded: 2 s, then status bit
 * 0 and no output) for every rank's result of the same call, and writes the
 * merged out (rows, C) bf16 and lse (rows,) with the sink. peers: host array
 * of the world buffers as mapped in this process (its own at [rank]). Every
 * rank must make the same sequence of calls with the same shape on its
 * buffer; calls on one stream are ordered, calls that overlap on several
 * streams race on the buffer. The call count lives in the buffer, so the
 * call can be replayed from a CUDA graph.
 */
size_t wpt_peer_bytes(int world, int64_t rows, int C);
int wpt_peer_alloc(size_t bytes, void** buffer, void* handle);
int wpt_peer_open(const void* handle, void** buffer);
int wpt_peer_close(void* buffer, int opened);
int wpt_attn_exchange(const float* part_o, const float* part_lse, int splits, int64_t rows, int H, int C,
                      const float* sink, void* const* peers, int world, int rank, void* out, float* lse,
                      void* stream);

/*
 * The output head's product ahead of sampling: scores (R, V) fp32 =
 * h (R, D) W (V, D)^T, bf16 inputs with fp32 accumulation on the tensor
 * cores (the vocabulary rows as the MMA's M, W streamed once). Replaces the
 * head call of a decode step (packages/wpt-model/src/wpt_model/model.py:267,
 * 471: nn.Linear(d_model, vocab, bias=False), bf16 under autocast, widened
 * with .float()), whose scores then feed wpt_accept's statistics and draw
 * (wpt_inference/__init__.py:173-182).
 *   h          bf16 (R, D), row stride h_stride elements (a multiple of 8)
 *   w          bf16 (V, D), row stride w_stride elements (a multiple of 8)
 *   D          a multiple of 64
 *   round_bf16 1: each score rounded to bf16 first, as the reference's
 *              autocast head returns it
 *   scores     fp32 (R, V), contiguous
 */
int wpt_head_scores(const void* h, int64_t h_stride, const void* w, int64_t w_stride, int R, int D, int V,
                    int round_bf16, float* scores, void* stream);

/*
 * The acceptance step of speculative decoding, WPT's rule
 * (packages/wpt-inference/src/wpt_inference/__init__.py:173-179 the
 * probabilities, :210-222 the loop), for R rows at once:
 *   p_j = softmax(mask(scores[i, j] / temperature)), the mask keeping the
 *         top_k largest (ties kept) when top_k > 0;
 *   draft j of row i is kept iff uniforms[i, j] * q[i, j, tok] < p_j[tok];
 *   the first rejected draft is replaced by a token drawn from
 *   normalize(max(0, p_j - q[i, j])); a row that keeps all its drafts adds
 *   one drawn from p_{n_i}.
 * The reference draws with torch.rand and torch.multinomial; here the draws
 * are explicit: uniforms (R, n) for the tests and resample (R,) for the
 * last token, which is the first index whose float64 running sum of the
 * weights exceeds resample[i] times their total.
 *   scores    fp32 (R, n + 1, V) target logits at each draft's place and one after
 *   drafted   int64 (R, n);  q  fp32 (R, n, V) the drafter's probabilities
 *   lengths   int64 (R,) drafts verified per row, or NULL for n
 *   scratch   caller scratch of wpt_accept_scratch_bytes(R, n, V) bytes, 16-byte
 *             aligned (segment statistics, chunk sums, per-row counters)
 *   tokens    int64 (R, n + 1): kept drafts then the drawn token, -1 padded
 *   accepted  int64 (R,): drafts kept per row
 */
int wpt_accept(const float* scores, const int64_t* drafted, const float* q, const float* uniforms,
               const float* resample, const int64_t* lengths, void* scratch, int64_t* tokens, int64_t* accepted,
               int R, int n, int V, float temperature, int top_k, void* stream);

/*
 * Ancestor masks of draft trees, the tree_bits argument of wpt_attn_prefill:
 * parents int64 (B, n) at row stride parents_stride_b (0: one (n,) tree for
 * every row), -1 for a root (a child of the last cache row) and
 * parents[b][i] < i otherwise; bits uint64 (B, n), bit j of bits[b][i] set
 * when node j is i or one of its ancestors. n <= 64. With positions (B, n)
 * int64 not NULL, also positions[b][i] = base[b] + i (node i's table row).
 * Computed on the device so that verification needs no host
 * synchronisation. Generalises the chain of drafts that WPT verifies
 * (packages/wpt-inference/src/wpt_inference/__init__.py:207, parents[i] =
 * i - 1) to a tree, with dense_attention's visible-mask semantics
 * (attention.py:74-82).
 */
int wpt_tree_bits(const int64_t* parents, int64_t parents_stride_b, int B, int n, uint64_t* bits,
                  const int64_t* base, int64_t* positions, void* stream);

/*
 * The generation cache's entries write (packages/wpt-model/src/wpt_model/
 * cache.py:110-128, Reading.everything's index put): row b's new entries
 * src[b, j] for j < counts[b] go to dst[b, first[b] + j]; entries past a
 * row's count are padding and are not written. One launch, no host
 * synchronisation (the reference reads the table's size and the written
 * rows back to the host first). Strides are in BYTES; rows of row_bytes
 * (a multiple of 16, any dtype), 16-byte aligned bases and strides. A
 * destination row at or past `capacity` is not written and sets the status
 * word's shape bit (bit 1).
 */
int wpt_cache_append(const void* src, int64_t src_stride_b, int64_t src_stride_n, void* dst, int64_t dst_stride_b,
                     int64_t dst_stride_n, const int64_t* first, const int64_t* counts, int B, int n, int row_bytes,
                     int64_t capacity, void* stream);

/* Bytes of scratch wpt_accept needs for R rows of n drafts over V entries
 * (0 for a bad shape). */
size_t wpt_accept_scratch_bytes(int R, int n, int V);

/* out[i] = x[i] / temperature as the acceptance kernels compute it (the
 * reference's float32 `scores / temperature`, wpt_inference/__init__.py:174):
 * exposed so that tests can compare it with IEEE division. fp32, n entries. */
int wpt_temperature_scale(const float* x, int64_t n, float temperature, float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WPT_ATTN_H_ */
