/*
 * b2a.h -- C ABI of the B200 attention hot path (libb2a.so).
 *
 * Replaces the attention / KV-cache operator surface of abho7/llm-inference-webgpu:
 *   CPU  groupedAttention   src/core/attention.js:32-66
 *        kvHeadFor          src/core/attention.js:74-76
 *        ropeFrequencies    src/core/ops.js:99-104
 *        ropeTables         src/core/ops.js:123-136
 *        ropeInPlace        src/core/ops.js:147-158
 *        KVCache            src/cpu/cache.js:18-119
 *   GPU  GpuKVCache         src/gpu/model.js:69-84
 *        rope-q, rope-k, KV append, ATTENTION dispatch sequence
 *                           src/gpu/model.js:323-346 (kernels ROPE src/gpu/kernels.js:360-389,
 *                           ATTENTION src/gpu/kernels.js:404-499)
 *
 * Conventions
 *   - Every call returns a b2a_status; b2a_last_error() holds the message of
 *     the calling thread's last failure. No call aborts, traps or throws.
 *   - Plain pointers and sizes only. `flags` says where the data pointers of a
 *     compute call live: B2A_HOST (default: staged through pinned buffers; the
 *     call returns after the results are back on the host, like the reference's
 *     readback, src/gpu/device.js:253-270) or B2A_DEVICE (zero-copy device
 *     pointers; the call only enqueues work on the context's stream).
 *   - A context is not re-entrant (src/gpu/model.js:231): a call made while
 *     another call on the same context is running returns B2A_EBUSY.
 *   - Tensor layouts: q [tokens][num_heads][head_dim]; new keys/values
 *     [tokens][num_kv_heads][head_dim] (== the reference's [seq, kvDim] rows);
 *     the device KV cache is head-major, per sequence and layer
 *     [kv_head][position][head_dim] (== KVCache.present(), src/cpu/cache.js:97-115).
 *   - Query head h reads KV head h / (num_heads / num_kv_heads) (blocked map).
 *   - RoPE is the half-split rotation at ABSOLUTE positions (src/cpu/model.js:103-113),
 *     evaluated in f64 from an f64 cos/sin table built on the host, stored to
 *     f32, then rounded to the cache dtype; cache bytes are bit-exact against
 *     the reference's f32 CPU path rounded the same way.
 */
#ifndef B2A_H
#define B2A_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2A_ABI_VERSION 1

typedef enum b2a_status {
  B2A_OK = 0,
  B2A_EINVAL = 1,     /* bad argument (shape, dtype, null pointer)                  */
  B2A_ERANGE = 2,     /* capacity / position range: the reference's RangeError      */
  B2A_EBUSY = 3,      /* context already running a call (src/gpu/model.js:231)      */
  B2A_ECUDA = 4,      /* CUDA runtime error (message in b2a_last_error)             */
  B2A_ENCCL = 5,      /* collective error                                           */
  B2A_ETIMEDOUT = 6,  /* a bounded device-side wait gave up                         */
  B2A_ENODEV = 7      /* no usable CUDA device                                      */
} b2a_status;

typedef enum b2a_dtype { B2A_F32 = 0, B2A_F16 = 1, B2A_BF16 = 2 } b2a_dtype;

enum { B2A_HOST = 0, B2A_DEVICE = 1 };

typedef struct b2a_ctx b2a_ctx;
typedef struct b2a_rope b2a_rope;
typedef struct b2a_kvcache b2a_kvcache;

/* ---- errors and version ------------------------------------------------- */
const char* b2a_last_error(void);
const char* b2a_status_name(b2a_status s);
int b2a_abi_version(void);

/* ---- context: one device, one stream (the reference's GpuContext, src/gpu/device.js:21) */
b2a_status b2a_init(int device, b2a_ctx** out);
b2a_status b2a_destroy(b2a_ctx* ctx);
/* Run subsequent work on an external cudaStream_t (NULL: the context's own). */
b2a_status b2a_set_stream(b2a_ctx* ctx, void* cuda_stream);
b2a_status b2a_synchronize(b2a_ctx* ctx);

/* ---- per-kernel device timing (GpuContext.timed, src/gpu/device.js:301-338) --
 * While enabled, every kernel the context launches is bracketed by CUDA events
 * on its stream. b2a_timing_read waits for the stream, then reports per kernel
 * kind the launch count and summed device milliseconds since the last read,
 * and clears them. */
typedef struct b2a_kernel_time {
  char name[32];
  int launches;
  double total_ms;
} b2a_kernel_time;
b2a_status b2a_timing_enable(b2a_ctx* ctx, int enable);
b2a_status b2a_timing_read(b2a_ctx* ctx, b2a_kernel_time* out, int max_entries, int* n_entries);

/* ---- host-side helpers (no device work) ---------------------------------- */
/* kvHeadFor, src/core/attention.js:74-76. Returns -1 for an invalid grouping. */
int b2a_kv_head_for(int query_head, int num_heads, int num_kv_heads);
/* ropeFrequencies, src/core/ops.js:99-104: inv_freq[head_dim/2] in f64. */
b2a_status b2a_rope_frequencies(int head_dim, double theta, double* inv_freq);
/* ropeTables, src/core/ops.js:123-136: f32 cos/sin [positions][head_dim/2]. */
b2a_status b2a_rope_tables(int head_dim, double theta, int positions, float* cos_out, float* sin_out);

/* ---- device RoPE table (the model's ropeTable, src/gpu/model.js:200-205) -- */
/* f64 cos/sin for positions 0..max_positions-1, kept on the device. */
b2a_status b2a_rope_create(b2a_ctx* ctx, int head_dim, double theta, int max_positions, b2a_rope** out);
b2a_status b2a_rope_destroy(b2a_rope* rope);

/* ---- KV cache (KVCache src/cpu/cache.js:18-119; GpuKVCache src/gpu/model.js:69-84) */
/* One device pool for keys and one for values, laid out
 * [batch][num_layers][num_kv_heads][capacity][head_dim] in `dtype`, zero-filled.
 * Each of the `batch` sequences has its own length. capacity < 1 fails with
 * B2A_ERANGE "cache capacity must be a positive integer, got N" (cache.js:24-26). */
b2a_status b2a_kvcache_create(b2a_ctx* ctx, int num_layers, int num_kv_heads, int head_dim,
                              int capacity, int batch, b2a_dtype dtype, b2a_kvcache** out);
b2a_status b2a_kvcache_destroy(b2a_kvcache* cache);
/* allocate(count), cache.js:52-60: returns where `count` new positions of
 * sequence `seq_idx` start, or B2A_ERANGE "cache holds L of C positions;
 * cannot add K more" without changing anything. */
b2a_status b2a_kvcache_allocate(b2a_kvcache* cache, int seq_idx, int count, int* at);
/* commit(count), cache.js:84-86. seq_idx -1 commits every sequence. */
b2a_status b2a_kvcache_commit(b2a_kvcache* cache, int seq_idx, int count);
/* length, cache.js:38. */
b2a_status b2a_kvcache_length(const b2a_kvcache* cache, int seq_idx, int* length);
/* Set every sequence's length at once (a cache filled by other means, e.g. a
 * benchmark or a restore). Each length must be within [0, capacity]. */
b2a_status b2a_kvcache_set_lengths(b2a_kvcache* cache, const int32_t* lengths);
/* reset(), cache.js:118. seq_idx -1 resets every sequence. */
b2a_status b2a_kvcache_reset(b2a_kvcache* cache, int seq_idx);
/* byteLength, cache.js:41-43 (in the cache's own dtype). */
b2a_status b2a_kvcache_byte_length(const b2a_kvcache* cache, size_t* bytes);
/* Device pools and element strides, for zero-copy callers:
 * strides[0..3] = elements between sequences, layers, kv heads, positions. */
b2a_status b2a_kvcache_pools(const b2a_kvcache* cache, void** keys, void** values, int64_t strides[4]);
/* writeAt(layer, at, keys, values, count), cache.js:63-67: raw store (no RoPE)
 * of `count` position-major rows [count][num_kv_heads*head_dim] in src_dtype,
 * rounded to the cache dtype. Positions at..at+count-1 must be < capacity. */
b2a_status b2a_kvcache_write_at(b2a_ctx* ctx, b2a_kvcache* cache, int layer, int seq_idx, int at,
                                const void* keys, const void* values, b2a_dtype src_dtype,
                                int count, int flags);
/* keysUpTo/valuesUpTo/present, cache.js:75-115: the first n positions of a
 * layer in present() layout [num_kv_heads][n][head_dim], raw cache dtype. */
b2a_status b2a_kvcache_read(b2a_ctx* ctx, const b2a_kvcache* cache, int layer, int seq_idx, int n,
                            void* keys_out, void* values_out, int flags);

/* ---- paged KV cache --------------------------------------------------------
 * The same cache object and operations, the storage split into pages: the pools
 * hold num_pages pages of page_size positions (plus one scratch page), each page
 * [num_layers][num_kv_heads][page_size][head_dim], and every sequence has a
 * page table mapping position p to page table[p / page_size], row p % page_size.
 * Sequences take pages from the shared pool as they grow (allocate, commit,
 * set_lengths, write_at, append and the attention calls that append) and give
 * them back on reset, so a batch of sequences of very different lengths needs
 * pool memory for the positions it holds, not batch x capacity. capacity stays
 * the per-sequence bound of the reference's KVCache (cache.js:24-26, 53-58).
 * page_size: a power of two, at least 128 (a 128-position tile of the attention
 * kernels never crosses a page). When the pool cannot back a call's new
 * positions the call fails with B2A_ERANGE "page pool exhausted: U of N pages in
 * use; sequence S needs K more" and no page of that call is taken. Pages of
 * positions beyond a sequence's mapped pages read as zeros. A paged cache's
 * allocate enqueues its page-table update on the owning context's stream, so,
 * unlike a contiguous cache's, it returns B2A_EBUSY while a call runs there. */
b2a_status b2a_kvcache_create_paged(b2a_ctx* ctx, int num_layers, int num_kv_heads, int head_dim,
                                    int capacity, int batch, b2a_dtype dtype, int page_size,
                                    int num_pages, b2a_kvcache** out);
/* The pages of sequence seq_idx in position order (up to max_entries of them)
 * and how many are mapped. For a paged cache b2a_kvcache_pools' strides[0] is
 * the page stride: element (layer, h, p) of the sequence is at
 * pages[p / page_size]*strides[0] + layer*strides[1] + h*strides[2] + (p % page_size)*strides[3].
 * A contiguous cache reports no pages (*mapped = 0). */
b2a_status b2a_kvcache_page_table(const b2a_kvcache* cache, int seq_idx, int32_t* pages_out, int max_entries,
                                  int* mapped);
/* Pages of the pool not held by any sequence (0 for a contiguous cache). */
b2a_status b2a_kvcache_free_pages(const b2a_kvcache* cache, int* free_pages);

/* The host page allocator of a paged cache, on its own (no device memory): it
 * keeps the page tables and the free pages. reserve maps pages until positions
 * [0, positions) of the sequence are backed (all or nothing); release returns a
 * sequence's pages (seq_idx -1: every sequence); the next reserve takes the most
 * recently released page first. */
typedef struct b2a_pagepool b2a_pagepool;
b2a_status b2a_pagepool_create(int num_pages, int page_size, int batch, int capacity, b2a_pagepool** out);
b2a_status b2a_pagepool_destroy(b2a_pagepool* pool);
b2a_status b2a_pagepool_reserve(b2a_pagepool* pool, int seq_idx, int positions);
b2a_status b2a_pagepool_release(b2a_pagepool* pool, int seq_idx);
b2a_status b2a_pagepool_table(const b2a_pagepool* pool, int seq_idx, int32_t* pages_out, int max_entries,
                              int* mapped);
b2a_status b2a_pagepool_free_pages(const b2a_pagepool* pool, int* free_pages);

/* ---- fused RoPE(K) + round + append (src/cpu/model.js:103-116; src/gpu/model.js:327-338) */
/* For sequence seq_idx with length L: rotate each KV head of k[t] at absolute
 * position L+t, round to the cache dtype and store it, and store v[t], at
 * cache position L+t, t < count. Length is unchanged until commit. */
b2a_status b2a_append_rope(b2a_ctx* ctx, b2a_kvcache* cache, const b2a_rope* rope, int layer,
                           int seq_idx, const void* k, const void* v, b2a_dtype src_dtype,
                           int count, int flags);

/* ---- single-token decode over every sequence of the cache ------------------
 * groupedAttention with seq=1, past=L_b (attention.js:32-66), preceded by the
 * rope-q / rope-k / append steps (src/gpu/model.js:327-338), fused.
 * For each sequence b (length L_b) and each layer in [layer_begin, layer_begin+num_layers):
 *   q rotated at position L_b; if k_new/v_new are given, k_new rotated at L_b
 *   and stored with v_new at cache position L_b; attention over positions 0..L_b.
 * q [batch][num_layers][num_heads][head_dim] (in_dtype);
 * k_new, v_new [batch][num_layers][num_kv_heads][head_dim] (in_dtype) or NULL
 *   (then position L_b must already hold the new key/value);
 * out [batch][num_layers][num_heads][head_dim] (out_dtype).
 * Lengths are not advanced (commit after the last layer, as the reference does). */
b2a_status b2a_attention_decode(b2a_ctx* ctx, b2a_kvcache* cache, const b2a_rope* rope,
                                int layer_begin, int num_layers, int num_heads,
                                const void* q, const void* k_new, const void* v_new,
                                b2a_dtype in_dtype, void* out, b2a_dtype out_dtype, int flags);

/* ---- host-pointer decode that returns before the results are back ----------
 * b2a_attention_decode with B2A_HOST pointers and the same layouts and
 * results, except that the call only enqueues the work: the uploads of q and
 * the new keys/values, the attention kernels and the download of `out`. The
 * reference's readback (src/gpu/device.js:253-270) makes every step wait for
 * its results; a serving loop that keeps its own host buffers can instead let
 * consecutive steps overlap on the GPU (one step's uploads and downloads run
 * under its neighbours' kernels; two device staging slots are used in turn).
 * Until b2a_synchronize(ctx) returns, the caller must not change q, k_new or
 * v_new nor read `out` of any call made since the last synchronisation (use
 * separate host buffers for calls in flight). Pinned host memory keeps the
 * copies asynchronous. A device-side wait that gave up is reported by
 * b2a_synchronize. */
b2a_status b2a_attention_decode_host_async(b2a_ctx* ctx, b2a_kvcache* cache, const b2a_rope* rope,
                                           int layer_begin, int num_layers, int num_heads,
                                           const void* q, const void* k_new, const void* v_new,
                                           b2a_dtype in_dtype, void* out, b2a_dtype out_dtype);

/* ---- decode that allocates nothing ------------------------------------------
 * No counterpart in the reference: its engine owns its WebGPU buffers itself.
 * Same work and arguments as b2a_attention_decode, for callers that cannot
 * allocate device memory: a server that has already handed the GPU's memory
 * to its own pools, or a caller running several streams that must not be
 * stalled by the device-wide synchronization cudaMalloc/cudaFree can cause.
 * Results agree with b2a_attention_decode within the split-KV merge's
 * rounding, not bit for bit (its chunk sizes may differ).
 * All pointers are device pointers (nothing is staged); the call only enqueues
 * work on the context's stream and never calls cudaMalloc or cudaFree.
 * The split-KV partials go to one fixed device array of
 * B2A_NOALLOC_SCRATCH_BYTES. b2a_init makes it resident on the context's GPU
 * (by looking up its address) and loads the kernels this call launches, so
 * create contexts before filling the GPU's memory; the GPU then holds the
 * array until the process exits. A call whose partials would not fit returns
 * B2A_ERANGE. All calls on a device share that array: calls that overlap on
 * the GPU race and corrupt each other, so order them (e.g. one stream). */
#define B2A_NOALLOC_SCRATCH_BYTES (16 * 1024 * 1024)
b2a_status b2a_attention_decode_noalloc(b2a_ctx* ctx, b2a_kvcache* cache, const b2a_rope* rope,
                                        int layer_begin, int num_layers, int num_heads,
                                        const void* q, const void* k_new, const void* v_new,
                                        b2a_dtype in_dtype, void* out, b2a_dtype out_dtype);

/* ---- causal prefill of one sequence ----------------------------------------
 * groupedAttention with seq=count, past=L (attention.js:32-66) for sequence
 * seq_idx, with RoPE on q and k at absolute positions L..L+count-1 and the K/V
 * append (src/cpu/model.js:103-123) fused in.
 * q [count][num_heads][head_dim]; k, v [count][num_kv_heads][head_dim] (in_dtype);
 * out [count][num_heads][head_dim] (out_dtype). */
b2a_status b2a_attention_prefill(b2a_ctx* ctx, b2a_kvcache* cache, const b2a_rope* rope,
                                 int layer, int seq_idx, int num_heads,
                                 const void* q, const void* k, const void* v, b2a_dtype in_dtype,
                                 int count, void* out, b2a_dtype out_dtype, int flags);

/* The prefill of `nseq` sequences (seq_begin, seq_begin+1, ...) in one call,
 * `count` new tokens each at that sequence's own cache length: q
 * [nseq][count][num_heads][head_dim], k and v [nseq][count][num_kv_heads][head_dim],
 * out [nseq][count][num_heads][head_dim]; the same arithmetic as nseq calls of
 * b2a_attention_prefill, in one append launch and one attention launch (many
 * short prompts fill the GPU together; no reference counterpart, the reference
 * runs one sequence at a time). Every sequence is checked as
 * b2a_attention_prefill checks it. */
b2a_status b2a_attention_prefill_batch(b2a_ctx* ctx, b2a_kvcache* cache, const b2a_rope* rope, int layer,
                                       int seq_begin, int nseq, int num_heads, const void* q, const void* k,
                                       const void* v, b2a_dtype in_dtype, int count, void* out, b2a_dtype out_dtype,
                                       int flags);

/* ---- the literal drop-in for groupedAttention (src/core/attention.js:32) ---
 * Same arguments and layouts as the JS: q [seq][num_heads*head_dim], keys and
 * values [past+seq][num_kv_heads*head_dim], out [seq][num_heads*head_dim], all
 * f32; q is already rotated and keys hold the rotated cache. `scores` is the
 * reference's scratch and is not used (may be NULL). head_dim <= 256. */
b2a_status b2a_grouped_attention(b2a_ctx* ctx, const float* q, const float* keys, const float* values,
                                 float* out, float* scores, int seq, int past, int num_heads,
                                 int num_kv_heads, int head_dim, int flags);

/* ---- split-KV decode across devices (one process per GPU) -------------------
 * Partial attention of one new token per sequence over the positions this
 * rank's cache holds: local positions [0, L_b) plus, when k_new/v_new are
 * given, the new token appended at local position L_b. q and k_new are rotated
 * at ABSOLUTE position q_positions[b] (host or device per flags).
 * partial [batch][num_heads][head_dim + 4] f32: the unnormalised output
 * sum_s 2^(t_s - m) v_s in [0, head_dim), then m (base-2 units of the scaled
 * score t = score*log2(e)) at head_dim and l = sum_s 2^(t_s - m) at head_dim+1.
 * An empty range gives l = 0, m = -inf. */
b2a_status b2a_attention_decode_partial(b2a_ctx* ctx, b2a_kvcache* cache, const b2a_rope* rope,
                                        int layer, int num_heads, const void* q,
                                        const void* k_new, const void* v_new, b2a_dtype in_dtype,
                                        const int32_t* q_positions, float* partial, int flags);
/* The same for layers [layer_begin, layer_begin + num_layers) in one launch
 * (the per-layer decode dispatch of src/gpu/model.js:323-346, one call per
 * decode step instead of one per layer): q [batch][num_layers][num_heads][64],
 * k_new/v_new [batch][num_layers][num_kv_heads][64], partial
 * [batch][num_layers][num_heads][head_dim + 4] (combine with
 * b2a_lse_combine as batch * num_layers rows). */
b2a_status b2a_attention_decode_partial_layers(b2a_ctx* ctx, b2a_kvcache* cache, const b2a_rope* rope,
                                               int layer_begin, int num_layers, int num_heads, const void* q,
                                               const void* k_new, const void* v_new, b2a_dtype in_dtype,
                                               const int32_t* q_positions, float* partial, int flags);
/* Log-sum-exp combine of `num_parts` partials laid out [num_parts][batch][num_heads][head_dim+4]
 * in ascending part order, into out [batch][num_heads][head_dim] (out_dtype). */
b2a_status b2a_lse_combine(b2a_ctx* ctx, const float* partials, int num_parts, int batch,
                           int num_heads, int head_dim, void* out, b2a_dtype out_dtype, int flags);
/* Split-KV decode over NCCL in one call (the per-layer decode dispatch of
 * src/gpu/model.js:323-346 with each rank holding a contiguous slice of every
 * sequence's positions; the reference itself runs on one device): this rank's
 * partials (b2a_attention_decode_partial_layers, written into its slot of a
 * per-context [world][batch][num_layers][num_heads][head_dim + 4] buffer), an
 * in-place ncclAllGather of the slots on the context's stream through the
 * caller's communicator `nccl_comm` (an ncclComm_t of `world` ranks in which
 * this process is `rank`), then b2a_lse_combine of the world slots in
 * ascending rank order into out [batch][num_layers][num_heads][head_dim]
 * (out_dtype; the same bits on every rank). Every rank passes the same q and
 * q_positions; k_new/v_new are appended and attended by rank world - 1 only
 * (the slice that ends the sequences) and ignored elsewhere. Device pointers
 * only (flags B2A_DEVICE). NCCL is loaded at the first call (libnccl.so.2,
 * the instance the process has loaded when there is one); B2A_ENCCL when it
 * cannot be loaded or the all-gather fails. Every rank must make the call,
 * the same number of times, in the same order as its other collectives. */
b2a_status b2a_split_kv_decode_nccl(b2a_ctx* ctx, b2a_kvcache* cache, const b2a_rope* rope, int layer_begin,
                                    int num_layers, int num_heads, const void* q, const void* k_new,
                                    const void* v_new, b2a_dtype in_dtype, const int32_t* q_positions,
                                    void* nccl_comm, int world, int rank, void* out, b2a_dtype out_dtype,
                                    int flags);

/* ---- projections either side of attention: int8 weights, per-row scales -----
 * The Qwen2.5 layer's q/k/v and output projections (src/cpu/model.js:98-101,
 * 125-128) over matVec (src/core/ops.js:33-41) with the reference's symmetric
 * per-channel int8 weights (src/core/quantize.js:36-67). */
/* Host, no device: quantizeInt8PerChannel. scales[r] = max|w[r][:]| / 127 (f32),
 * codes = round-half-away-from-zero(w / scale) clamped to [-127, 127]; an
 * all-zero row gets scale 0 and zero codes. */
b2a_status b2a_quantize_int8_per_channel(const float* w, int rows, int cols, int8_t* codes, float* scales);
/* out[t][r] = residual[t][r] + scales[r] * sum_c codes[r][c] * x[t][c] + bias[r],
 * t < tokens: codes [rows][cols] (cols a multiple of 16; 16-byte aligned on the
 * device), scales and bias [rows] in their dtypes (bias, residual may be NULL),
 * x [tokens][cols] (16-byte aligned rows on the device), out and residual
 * [tokens][rows] in out_dtype. The residual add is o_proj's x += W·a. */
b2a_status b2a_linear_int8(b2a_ctx* ctx, const int8_t* codes, const void* scales, b2a_dtype scale_dtype,
                           const void* bias, b2a_dtype bias_dtype, const void* x, b2a_dtype x_dtype, int rows,
                           int cols, int tokens, const void* residual, void* out, b2a_dtype out_dtype, int flags);
/* The fused q/k/v projection: codes/scales/bias hold the q rows (q_rows =
 * num_heads*head_dim), then the k rows, then the v rows (kv_rows each);
 * q_out [tokens][q_rows], k_out and v_out [tokens][kv_rows] in out_dtype, the
 * layouts b2a_attention_decode / _prefill take for q, k_new and v_new. */
b2a_status b2a_qkv_int8(b2a_ctx* ctx, const int8_t* codes, const void* scales, b2a_dtype scale_dtype,
                        const void* bias, b2a_dtype bias_dtype, const void* x, b2a_dtype x_dtype, int hidden,
                        int q_rows, int kv_rows, int tokens, void* q_out, void* k_out, void* v_out,
                        b2a_dtype out_dtype, int flags);

/* ---- split-KV decode with the exchange fused into the attention kernel ------
 * No reference counterpart (the reference runs on one device). The merge is the
 * log-sum-exp combine of b2a_lse_combine, in ascending rank order, so every rank
 * writes the same bits.
 *
 * An exchange connects `world` (<= 8) processes, one GPU each, for caches of
 * `batch` sequences with num_heads query and num_kv_heads KV heads. Every rank
 * creates one, publishes its handle (b2a_exchange_handle, B2A_EXCHANGE_HANDLE_BYTES
 * bytes) to the others over any host channel and opens all of them in rank order
 * (b2a_exchange_open). Then every rank calls b2a_attention_decode_split once per
 * step, the same number of times: inside the attention kernel the last CTA of
 * each (sequence, KV head) stores the group's merged partial into every rank's
 * exchange buffer (peer stores over NVLink, each value tagged with the step
 * number in the same 64-bit word), waits (at most ~1 s) until all ranks' words
 * for the group carry the step and writes the combined, normalised output. A wait that gives up makes that call (host pointers) or the
 * next b2a_synchronize return B2A_ETIMEDOUT; recreate the exchange on every rank
 * after that. The cache's (sequence, KV head) groups must not outnumber the
 * CTAs that fit on the GPU at once (three per SM). */
typedef struct b2a_exchange b2a_exchange;
#define B2A_EXCHANGE_HANDLE_BYTES 64
b2a_status b2a_exchange_create(b2a_ctx* ctx, int world, int rank, int batch, int num_heads, int num_kv_heads,
                               b2a_exchange** out);
/* An exchange for calls that cover num_layers layers each
 * (b2a_attention_decode_split_layers); b2a_exchange_create is num_layers 1. */
b2a_status b2a_exchange_create_layers(b2a_ctx* ctx, int world, int rank, int batch, int num_layers,
                                      int num_heads, int num_kv_heads, b2a_exchange** out);
b2a_status b2a_exchange_handle(const b2a_exchange* ex, void* handle);
b2a_status b2a_exchange_open(b2a_exchange* ex, const void* handles);
/* Wires rank `peer` of ex to another exchange object of this process on the same
 * device, instead of an IPC handle (single-GPU tests of the timeout path). Two
 * ranks wired this way must never run their steps at the same time: kernels that
 * wait on each other cannot share one GPU. */
b2a_status b2a_exchange_connect_local(b2a_exchange* ex, int peer, const b2a_exchange* other);
b2a_status b2a_exchange_destroy(b2a_exchange* ex);
/* One decode step: like b2a_attention_decode_partial for this rank's positions
 * (k_new/v_new only on the rank holding the new token), then the exchange, with
 * out [batch][num_heads][head_dim] in out_dtype. f16 or bf16 caches. */
b2a_status b2a_attention_decode_split(b2a_ctx* ctx, b2a_kvcache* cache, const b2a_rope* rope, int layer,
                                      int num_heads, const void* q, const void* k_new, const void* v_new,
                                      b2a_dtype in_dtype, const int32_t* q_positions, b2a_exchange* ex,
                                      void* out, b2a_dtype out_dtype, int flags);
/* One decode step over layers [layer_begin, layer_begin + num_layers) in one
 * launch (the per-layer dispatch of src/gpu/model.js:323-346 folded into one
 * call): layouts as b2a_attention_decode_partial_layers, out
 * [batch][num_layers][num_heads][head_dim]; the exchange must have been made
 * for num_layers, and its (sequence, layer, KV head) groups must fit on the
 * GPU at once (three CTAs per SM). */
b2a_status b2a_attention_decode_split_layers(b2a_ctx* ctx, b2a_kvcache* cache, const b2a_rope* rope,
                                             int layer_begin, int num_layers, int num_heads, const void* q,
                                             const void* k_new, const void* v_new, b2a_dtype in_dtype,
                                             const int32_t* q_positions, b2a_exchange* ex, void* out,
                                             b2a_dtype out_dtype, int flags);

/* ---- the Qwen2 decoder around the attention path ------------------------------
 * ReferenceModel.forward / generate (src/cpu/model.js:55-187) and
 * GpuModel.forward (src/gpu/model.js:227-400) over int8 weights with one scale
 * per output row. One layer, in the order it runs:
 *   h = x + O(attn(RoPE(Q(rms(x))), RoPE(K(rms(x))), V(rms(x))))
 *   y = h + Down(silu(Gate(rms(h))) * Up(rms(h)))
 * then the final RMSNorm and the tied output projection (the embedding rows).
 * A model owns its weights on the device, a one-sequence f16 KV cache of
 * `capacity` positions, the RoPE table (max_positions entries) and its
 * activations; q/k/v reach attention as f16, everything else is f32. */
typedef struct b2a_model b2a_model;
typedef struct b2a_model_config {
  int hidden_size;         /* num_heads * 64                                   */
  int intermediate_size;   /* a multiple of 16                                 */
  int num_layers;
  int num_heads;
  int num_kv_heads;        /* divides num_heads, at most 8 query heads each    */
  int vocab_size;
  int max_positions;       /* max_position_embeddings: RoPE table entries      */
  double rope_theta;
  double rms_norm_eps;
  b2a_dtype scale_dtype;   /* dtype of every per-row scale: B2A_F16 or B2A_F32 */
} b2a_model_config;
/* One decoder layer's tensors (row-major, [out_features][in_features]). */
typedef struct b2a_layer_weights {
  const float* input_norm;       /* [hidden]                                          */
  const float* post_attn_norm;   /* [hidden]                                          */
  const int8_t* qkv;             /* [hidden + 2*kv_dim][hidden]: q rows, k rows, v rows */
  const void* qkv_scales;        /* [hidden + 2*kv_dim] in scale_dtype                */
  const float* qkv_bias;         /* [hidden + 2*kv_dim]                               */
  const int8_t* o;               /* [hidden][hidden]                                  */
  const void* o_scales;
  const int8_t* gate;            /* [intermediate][hidden]                            */
  const void* gate_scales;
  const int8_t* up;              /* [intermediate][hidden]                            */
  const void* up_scales;
  const int8_t* down;            /* [hidden][intermediate]                            */
  const void* down_scales;
} b2a_layer_weights;
b2a_status b2a_model_create(b2a_ctx* ctx, const b2a_model_config* cfg, int capacity, b2a_model** out);
b2a_status b2a_model_destroy(b2a_model* model);
/* Copies weights in from host (B2A_HOST) or device (B2A_DEVICE) memory. Every
 * layer, the embedding and the final norm must be loaded before a forward. */
b2a_status b2a_model_load_layer(b2a_model* model, int layer, const b2a_layer_weights* w, int flags);
/* The tied embedding, codes [vocab][hidden] and scales [vocab]: the input
 * lookup dequantizes one row per token, the output projection is the int8
 * product with every row. */
b2a_status b2a_model_load_embedding(b2a_model* model, const int8_t* codes, const void* scales, int flags);
b2a_status b2a_model_load_final_norm(b2a_model* model, const float* weight, int flags);
/* ReferenceModel.forward(tokenIds, {cache}): runs `seq` tokens at positions
 * length..length+seq-1 of the model's cache, then commits them. logits
 * ([vocab] f32, the last position's; may be NULL) and next_token (the first
 * index of the largest logit; may be NULL) in the memory `flags` names, like
 * tokens. Errors as the reference: B2A_EINVAL "forward: need at least one
 * token", B2A_ERANGE for a token outside the vocabulary or a full cache. */
b2a_status b2a_model_forward(b2a_model* model, const int32_t* tokens, int seq, float* logits, int32_t* next_token,
                             int flags);
/* ReferenceModel.generate(promptIds, {maxTokens, stopTokens}), greedy, from an
 * empty cache: the prompt in one pass, then one pass per new token, each
 * token chosen and fed back on the device. Host arrays: tokens_out and
 * best_logits [max_tokens] (the chosen token's logit); *n_generated stops
 * short of max_tokens after a stop token (which is included). */
b2a_status b2a_model_generate(b2a_model* model, const int32_t* prompt, int n_prompt, int max_tokens,
                              const int32_t* stop_tokens, int n_stop, int32_t* tokens_out, float* best_logits,
                              int* n_generated);
/* How a one-token forward runs: B2A_DECODE_PERSISTENT (the default where the
 * shape fits: hidden <= 1024, intermediate <= 8192) is one cooperative kernel
 * per token for every layer, the output projection and the pick;
 * B2A_DECODE_LAYERED is the per-layer launches a multi-token forward uses. */
enum { B2A_DECODE_LAYERED = 0, B2A_DECODE_PERSISTENT = 1 };
b2a_status b2a_model_set_decode_path(b2a_model* model, int path);
b2a_status b2a_model_decode_path(const b2a_model* model, int* path);
b2a_status b2a_model_reset(b2a_model* model);

/* ---- weights: safetensors files (Safetensors, src/core/safetensors.js:36-199) -------
 * Opening reads and validates the header against the file's size with the
 * reference's checks and messages (B2A_EINVAL): "not a safetensors file",
 * "header length L does not fit in a N-byte file", "header is not valid UTF-8
 * JSON: ...", "NAME: unknown dtype ...", "NAME: shape must be an array of
 * non-negative integers", "NAME: data_offsets must be a pair", "NAME: bad
 * data_offsets [b, e]", "NAME: ends at E but the data section is only D bytes",
 * "NAME: shape [..] of DT needs X bytes but the header reserves Y", "B overlaps
 * A". Tensor bytes are read on demand (a file is pread, a memory image is
 * copied at open). Names come in the header's order. */
typedef struct b2a_safetensors b2a_safetensors;
b2a_status b2a_safetensors_open(const char* path, b2a_safetensors** out);
b2a_status b2a_safetensors_open_memory(const void* bytes, size_t size, b2a_safetensors** out);
b2a_status b2a_safetensors_close(b2a_safetensors* st);
int b2a_safetensors_count(const b2a_safetensors* st);
/* The index-th name (header order); NULL when out of range. Valid until close. */
const char* b2a_safetensors_name(const b2a_safetensors* st, int index);
/* The __metadata__ object as JSON text, or NULL when the header has none. */
const char* b2a_safetensors_metadata(const b2a_safetensors* st);
/* info(name): dtype ("F32", "BF16", ...; at least 16 chars of room), up to
 * max_dims dimensions, their count and the tensor's byte length. B2A_EINVAL
 * 'no tensor named "NAME"' for an unknown name. */
b2a_status b2a_safetensors_info(const b2a_safetensors* st, const char* name, char* dtype, int64_t* shape,
                                int max_dims, int* ndim, int64_t* byte_length);
/* readRaw: the tensor's bytes as stored (capacity >= byte_length). */
b2a_status b2a_safetensors_read_raw(const b2a_safetensors* st, const char* name, void* dst, size_t capacity);
/* readF32: widened to f32 (F32, BF16, F16, F64 rounded to nearest even);
 * "NAME: cannot widen DT to f32" otherwise. count >= the element count. */
b2a_status b2a_safetensors_read_f32(const b2a_safetensors* st, const char* name, float* dst, size_t count);
/* The model's weights from a Qwen2 checkpoint (GpuModel.load, src/gpu/model.js:147-207;
 * config.checkAgainst, src/core/config.js:125-150): the file must hold exactly
 * the tensors the model's config implies (tied embeddings: no lm_head.weight),
 * each with its shape, else B2A_EINVAL "weights do not match config (N
 * problems): ...". Every matrix is widened to f32, quantized to int8 per output
 * row (b2a_quantize_int8_per_channel; the scale then stored in the model's
 * scale dtype) and uploaded with the norms and q/k/v biases. */
b2a_status b2a_model_load_safetensors(b2a_model* model, const b2a_safetensors* st);
b2a_status b2a_model_length(const b2a_model* model, int* length);
/* The model's KV cache (layers x kv heads x capacity, f16), for reading the
 * present keys and values with b2a_kvcache_read. Owned by the model. */
b2a_status b2a_model_cache(b2a_model* model, b2a_kvcache** cache);

#ifdef __cplusplus
}
#endif
#endif /* B2A_H */
