// Internal declarations shared by the C ABI (api.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <atomic>
#include <cstdint>
#include <string>
#include <vector>

#include "b2a.h"

struct b2a_ctx {
  int device = 0;
  int sm_count = 148;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;        // where work is enqueued
  std::atomic<int> busy{0};
  // device staging for host-pointer calls, grown on demand
  void* d_stage = nullptr;
  size_t d_stage_bytes = 0;
  // split-KV partials, grown on demand
  void* d_scratch = nullptr;
  size_t d_scratch_bytes = 0;
  // rotated f16 queries of a tensor-core prefill call, grown on demand
  void* d_qrot = nullptr;
  size_t d_qrot_bytes = 0;
  int32_t* d_err = nullptr;             // device error word (bounded waits, bounds checks)
  int32_t* h_err = nullptr;             // pinned host copy of it, read after a call's stream sync
  int32_t* d_counters = nullptr;        // fused split-KV merge counters, kept zeroed
  size_t d_counters_bytes = 0;
  int32_t* d_positions = nullptr;       // staging for host q_positions
  int d_positions_cap = 0;
  // per-kernel timing (b2a_timing_enable / b2a_timing_read)
  bool timing = false;
  struct TimingRec {
    int kind;
    cudaEvent_t start, stop;
  };
  std::vector<TimingRec> timing_recs;
  std::vector<cudaEvent_t> event_pool;
  // host-pointer decode pipeline: uploads and downloads overlap the kernels
  cudaStream_t copy_in = nullptr;
  cudaStream_t copy_out = nullptr;
  std::vector<cudaEvent_t> pipe_events;
  // asynchronous host-pointer decode (b2a_attention_decode_host_async): two
  // staging slots used in turn, each free again once its event (recorded
  // after the slot's last download) has completed
  void* d_async[2] = {nullptr, nullptr};
  size_t d_async_bytes[2] = {0, 0};
  cudaEvent_t async_free[2] = {nullptr, nullptr};
  bool async_used[2] = {false, false};
  int async_next = 0;
};

namespace b2a {
// Kernel kinds reported by b2a_timing_read.
enum KernelKind { K_ATTN_SIMT = 0, K_ATTN_MMA, K_COMBINE, K_ROPE_APPEND, K_WRITE_AT, K_GROUPED, K_PREFILL_TC,
                  K_PREFILL_PAIR, K_LINEAR, K_EMBED, K_RMSNORM, K_SWIGLU, K_ARGMAX, K_DECODE_STEP, K_NUM_KINDS };
extern const char* const kKernelNames[K_NUM_KINDS];

// Brackets one launch with events on the context's stream while timing is on.
class KernelTimer {
 public:
  KernelTimer(b2a_ctx* ctx, int kind);
  void stop();
  ~KernelTimer() { stop(); }

 private:
  b2a_ctx* ctx_;
  int kind_;
  cudaEvent_t start_ = nullptr;
  bool done_ = false;
};
}  // namespace b2a

struct b2a_rope {
  b2a_ctx* ctx = nullptr;   // creating context; not used after creation
  int device = 0;
  int head_dim = 0;
  double theta = 0;
  int max_positions = 0;
  double* d_cos = nullptr;  // [max_positions][head_dim/2]
  double* d_sin = nullptr;
  float* d_cos32 = nullptr; // the same tables rounded to f32 (query rotation
  float* d_sin32 = nullptr; // ahead of a 16-bit tensor-core operand)
};

struct b2a_kvcache {
  b2a_ctx* ctx = nullptr;   // owning context: must outlive the cache for data calls
  int device = 0;
  int layers = 0, kv_heads = 0, head_dim = 0, capacity = 0, batch = 0;
  b2a_dtype dtype = B2A_F16;
  void* d_k = nullptr;
  void* d_v = nullptr;
  int32_t* d_len = nullptr;     // device mirror of len, updated in stream order
  std::vector<int32_t> len;     // committed length per sequence (host truth)
  int64_t s_seq = 0, s_layer = 0, s_head = 0;  // element strides; position stride = head_dim
  // 2D TMA views of the pools as [rows][head_dim] with 64-row boxes and
  // 128-byte swizzle (f16/bf16, head_dim 64); has_tmaps false otherwise
  bool has_tmaps = false;
  CUtensorMap tmap_k;
  CUtensorMap tmap_v;
  // Paged layout (page_size > 0): the pools hold num_pages + 1 pages of
  // page_size positions, each [layers][kv_heads][page_size][head_dim]; page
  // num_pages is a scratch page that every unmapped page-table entry names, so
  // no table entry ever points outside the pools. The strides above then
  // describe one page (s_seq = elements per page) and positions are page rows.
  int page_size = 0, page_shift = 0, num_pages = 0, max_pages = 0;
  int32_t* d_pages = nullptr;     // [batch][max_pages] device page table
  b2a_pagepool* pool = nullptr;   // host page tables and free pages
};

namespace b2a {

// ---- errors ----------------------------------------------------------------
b2a_status fail(b2a_status s, const char* fmt, ...);
b2a_status cuda_fail(cudaError_t e, const char* what);
inline size_t dtype_size(b2a_dtype d) { return d == B2A_F32 ? 4 : 2; }

// ---- kernel parameter blocks -------------------------------------------------
// Attention over a head-major cache: rows of queries (b, layer, t, head).
constexpr int kLenInline = 64;
constexpr int kMaxWorld = 8;   // ranks of a peer exchange

struct AttnParams {
  const void* kc;
  const void* vc;
  void* kc_w;                 // same pools, writable (fused append)
  void* vc_w;
  int64_t s_seq, s_layer, s_head;
  // paged cache: [cache batch][max_pages] page of each 2^page_shift positions
  // (s_seq is then the page stride); null for a contiguous cache
  const int32_t* pages;
  int max_pages, page_shift;
  int cache_dtype;
  const int32_t* len;         // [cache batch] past length per sequence (device)
  int seq_begin;              // first cache sequence of this call
  // the same lengths for this call's sequences, by value, when there are at
  // most kLenInline of them (n_len_inline = batch; 0: read len)
  int n_len_inline;
  int32_t len_inline[64];
  int batch, num_layers, layer_begin, tokens, heads, kv_heads, group, head_dim;
  const void* q;              // [batch][num_layers][tokens][heads][D]
  const void* k_new;          // [batch][num_layers][tokens][kv_heads][D] or null
  const void* v_new;
  int in_dtype;
  const int32_t* q_pos;       // absolute rope position per sequence (partials) or null
  int horizon_extra;          // decode/prefill: 1 (slot L+t inclusive); partial: (k_new?1:0)
  const double* rope_cos;
  const double* rope_sin;
  const float* rope_cos32;    // f32 copies, for queries rounded to 16 bits afterwards
  const float* rope_sin32;
  int rope_max;
  float* partial;             // [rows][nchunks][D+4]
  int chunk;                  // positions per chunk (multiple of 64)
  int nchunks;                // chunks per row (max over rows)
  int32_t* err;
  const void* tmap_k;         // host CUtensorMap* of the pools (tensor-core path), or null
  const void* tmap_v;
  // Prefill with an f16 cache: the append kernel also writes RoPE(q) as f16
  // rows [sequence][token][head][64] to q_rot (null: not asked for), and the
  // tensor-core prefill loads its query tiles from there through tmap_q (a
  // host CUtensorMap* over q_rot as [rows][heads * 64], 128-row boxes).
  uint16_t* q_rot;
  const void* tmap_q;
  // host CUtensorMap* of a prefill call's 16-bit output as [sequence][token]
  // [heads * 64] (128-row boxes), or null: the epilogue then stores by thread
  const void* tmap_o;
  // Fused split-KV merge (tensor-core path): when fuse_out is set, a group
  // whose keys fit one chunk writes its result straight to fuse_out, and the
  // last CTA of every other group merges that group's chunk partials, so no
  // separate combine launch is needed. fuse_mode 0: normalised output
  // [rows][D] in fuse_dtype; 1: merged partial [rows][D+4] f32. counters: one
  // zeroed int per (sequence, layer, KV head) of the call, left zeroed.
  void* fuse_out;
  int fuse_dtype;
  int fuse_mode;
  int32_t* counters;
  // fuse_mode 2 (split-KV across ranks): each group's merged partial is stored
  // into every rank's exchange buffer, x_peer[r] = [2 parities][world][x_rows]
  // [D+4] words of 64 bits, each holding one f32 value in its low half and the
  // step number in its high half (a reader spins on the words themselves, no
  // separate flag); the group's last CTA then waits for all ranks' words in
  // its own buffer (x_local) and writes the combined output to fuse_out.
  // x_epoch counts steps (bumped by the launch's last CTA, counted in x_done).
  uint64_t* x_peer[kMaxWorld];
  const uint64_t* x_local;
  int32_t* x_epoch;
  int32_t* x_done;
  int x_world, x_rank, x_rows;
};

// Projection with int8 weights (k_linear.cu): out[t][r] = residual[t][r] +
// scale[r] * sum_c w[r][c] x[t][c] + bias[r]. Output rows are split into up to
// three segments (q, k, v of a fused QKV weight): rows [seg_end[s-1], seg_end[s])
// go to out[s] as [tokens][rows of the segment].
struct LinearParams {
  const int8_t* w;            // [rows][cols], cols a multiple of 16
  const void* scale;          // [rows]
  int scale_dtype;
  const void* bias;           // [rows] or null
  int bias_dtype;
  const void* x;              // [tokens][cols]
  int x_dtype;
  int rows, cols, tokens;
  void* out[3];
  int seg_end[3];
  int nseg;
  int out_dtype;
  const void* residual;       // one segment only: [tokens][rows] in out_dtype, or null
};

struct CombineParams {
  const float* partial;       // chunked: [rows][nchunks][D+4]; cross-rank: [nchunks][rows][D+4]
  int64_t rows;
  int nchunks, head_dim;
  int part_stride_rows;       // 0: chunked layout; else rows between parts (cross-rank layout)
  void* out;                  // mode 0: [rows][D] in out_dtype; mode 1: merged partial [rows][D+4] f32
  int out_dtype;
  int mode;
  // chunked layout only: when len is set, row (b, layer, t, head) holds
  // max(1, ceil((len[seq_begin+b] + t + extra) / chunk)) valid chunks
  const int32_t* len;
  int seq_begin, chunk, extra, tokens, heads, num_layers;
};

// Element offset of (cache sequence bc, layer, kv head g, position pos) in the
// pools. Contiguous: sequence-major blocks of s_seq elements. Paged: the page
// that holds pos, then the row pos mod page size within it; a run of positions
// that starts at a multiple of 128 and stays under the next multiple of 128
// lies in one page, contiguous, exactly as in the contiguous layout.
__host__ __device__ inline int64_t kv_elem(const AttnParams& p, int bc, int layer, int g, int pos) {
  int64_t unit = bc;
  int off = pos;
  if (p.pages != nullptr) {
    unit = p.pages[static_cast<int64_t>(bc) * p.max_pages + (pos >> p.page_shift)];
    off = pos & ((1 << p.page_shift) - 1);
  }
  return unit * p.s_seq + static_cast<int64_t>(layer) * p.s_layer + static_cast<int64_t>(g) * p.s_head +
         static_cast<int64_t>(off) * p.head_dim;
}

// Past length of the call's sequence b (by value when the host passed it).
__host__ __device__ inline int len_of(const AttnParams& p, int b) {
  return b < p.n_len_inline ? p.len_inline[b] : p.len[p.seq_begin + b];
}

// RoPE(k) + append of `count` new keys/values for each of nseq sequences from seq_idx
// (k_new/v_new [nseq][count][kv_heads][D]) at each sequence's length
cudaError_t launch_rope_append(const AttnParams& p, int seq_idx, int count, cudaStream_t st, int nseq = 1);
cudaError_t launch_write_at(const b2a_kvcache* c, int layer, int seq_idx, int at, const void* k,
                            const void* v, int src_dtype, int count, cudaStream_t st);
cudaError_t launch_read(const b2a_kvcache* c, int layer, int seq_idx, int n, void* k_out, void* v_out,
                        cudaStream_t st);
cudaError_t launch_lengths_update(int32_t* d_len, int idx, int batch, int count, int mode, cudaStream_t st);
// the cache's pools, strides and page table in p (the rest of p untouched)
void fill_cache_params(AttnParams& p, const b2a_kvcache* c);

// ---- paged caches (pages.cu) --------------------------------------------------
// Entries of the device page table written by one launch, by value.
constexpr int kPageUpdateMax = 240;
struct PageUpdate {
  int n;
  int32_t idx[kPageUpdateMax];    // entry index seq * max_pages + k
  int32_t page[kPageUpdateMax];
};
cudaError_t launch_page_table_update(int32_t* table, const PageUpdate& u, cudaStream_t st);
// Backs positions [0, positions[i]) of sequences first..first+n-1 with pages
// (all or nothing: B2A_ERANGE "page pool exhausted ..." when the free pages do
// not cover every sequence's new pages) and updates the device table in stream
// order. A no-op for a contiguous cache. The caller holds the context.
b2a_status cache_reserve(b2a_kvcache* c, int first, int n, const int32_t* positions);
inline b2a_status cache_reserve1(b2a_kvcache* c, int seq, int positions) {
  const int32_t pos = positions;
  return cache_reserve(c, seq, 1, &pos);
}
// cache_reserve for every sequence of the cache, to its length + extra.
b2a_status cache_reserve_all(b2a_kvcache* c, int extra);
// Returns the pages of one sequence (seq -1: all) to the pool; no-op when contiguous.
b2a_status cache_release(b2a_kvcache* c, int seq);
// host page-pool access for the cache (pages.cu)
int pool_mapped(const b2a_pagepool* pool, int seq);
const int32_t* pool_row(const b2a_pagepool* pool, int seq);
cudaError_t launch_attn_simt(const AttnParams& p, cudaStream_t st);
bool attn_mma_supported(const AttnParams& p);
int64_t attn_mma_items(const AttnParams& p, const int32_t* host_len);
int attn_mma_max_fused_chunks();
cudaError_t launch_attn_mma(const AttnParams& p, int64_t items, cudaStream_t st);
cudaError_t launch_combine(const CombineParams& p, cudaStream_t st);
// Load a module's kernels onto the current device ahead of their first launch.
cudaError_t preload_attn_mma();
cudaError_t preload_attn_simt();
cudaError_t preload_pages();
// Called by b2a_init with `device` current: makes the no-alloc decode's scratch
// array and every kernel that decode launches resident on the device, so that
// later no-alloc calls need no device memory at all (noalloc.cu).
b2a_status noalloc_prepare(int device);
bool prefill_tc_supported(const AttnParams& p);
cudaError_t launch_prefill_tc(const AttnParams& p, void* out, int out_dtype, cudaStream_t st);
bool prefill_pair_supported(const AttnParams& p);
cudaError_t launch_prefill_pair(const AttnParams& p, void* out, int out_dtype, cudaStream_t st);
cudaError_t launch_linear_int8(const LinearParams& p, cudaStream_t st);
cudaError_t launch_grouped_generic(const float* q, const float* k, const float* v, float* out, int seq,
                                   int past, int heads, int kv_heads, int head_dim, cudaStream_t st);

// ---- the decoder around attention (k_model.cu, model.cu) -----------------------
constexpr int kErrBadToken = 16;   // error word: a device token outside the vocabulary
// x[t][:] = codes[tokens[t]][:] * scales[tokens[t]] (f32)
cudaError_t launch_embed_int8(const int32_t* tokens, int count, const int8_t* codes, const void* scales,
                              int scale_dtype, int hidden, int vocab, float* x, int32_t* err, cudaStream_t st);
// out[r][:] = RMSNorm(x[r][:]) * w, rows of `hidden` f32
cudaError_t launch_rmsnorm(const float* x, const float* w, double eps, int rows, int hidden, float* out,
                           cudaStream_t st);
// h[i] = silu(gu[2i]) * gu[2i+1]: gate and up outputs interleaved
cudaError_t launch_swiglu(const float* gu, float* h, int64_t n, cudaStream_t st);
// the first index of the largest of logits[0..n) -> *token (and its value ->
// *value); scratch: kArgmaxScratchBytes, its counter word zeroed once at
// allocation (the kernel leaves it zeroed)
constexpr size_t kArgmaxScratchBytes = 8192;
cudaError_t launch_argmax(const float* logits, int n, int32_t* token, float* value, void* scratch,
                          cudaStream_t st);

// ---- the whole-decoder decode step (k_decode_step.cu) ----------------------
// One layer's tensors as the step kernel reads them (device pointers).
struct StepLayer {
  const int8_t* qkv;      // [hidden + 2 kv_dim][hidden]
  const int8_t* o;        // [hidden][hidden]
  const int8_t* gu;       // [2 inter][hidden]: gate row i at 2i, up row i at 2i+1
  const int8_t* down;     // [hidden][inter]
  const void* s_qkv;
  const void* s_o;
  const void* s_gu;
  const void* s_down;
  const float* b_qkv;
  const float* n_in;
  const float* n_post;
};
struct StepParams {
  const StepLayer* layers;                 // device array [num_layers]
  int num_layers, hidden, inter, heads, kv_heads, vocab, scale_dtype;
  double eps;
  const int8_t* emb;                       // tied embedding [vocab][hidden] and its scales
  const void* s_emb;
  const float* n_final;
  uint16_t* kc;                            // one sequence's f16 cache: [layer][kv head][pos][64]
  uint16_t* vc;
  int64_t s_layer, s_head;
  int past;                                // keys already cached; the new token goes to `past`
  const double* rope_cos;                  // [max_positions][32]
  const double* rope_sin;
  const int32_t* token_in;
  int32_t* token_out;
  float* best_out;                         // the chosen token's logit, or null
  unsigned long long* key;                 // argmax word of this step, zero on entry
  float* logits;                           // [vocab]
  float* x;                                // scratch: [hidden], [hidden + 2 kv_dim], partials, [inter]
  float* qkv;
  float* part;
  float* h;
  unsigned* bar;                           // grid-barrier arrival counter
  unsigned bar_base;                       // its value at launch
  int* abort;                              // set by a CTA whose barrier wait gave up
  int32_t* err;
  int32_t* len;                            // device cache length, set to past + 1
  int attn_chunk, attn_nchunks;            // attention items: heads x chunks of attn_chunk keys (<= 128)
};
size_t decode_step_smem_bytes();
int decode_step_barriers(int num_layers);
int decode_step_attn_chunk();   // keys per attention item
bool decode_step_supported(int hidden, int inter, int q_rows, int vocab, int ctas);
int decode_step_max_ctas();
cudaError_t launch_decode_step(const StepParams& p, int ctas, cudaStream_t st);

// Device-pointer bodies of b2a_attention_decode (one layer) and
// b2a_attention_prefill: the caller validated the shapes and holds the context.
b2a_status attn_decode_device(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope, int layer, int num_heads,
                              const void* q, const void* k_new, const void* v_new, b2a_dtype in_dtype, void* out,
                              b2a_dtype out_dtype);
b2a_status attn_prefill_device(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope, int layer, int seq_idx,
                               int num_heads, const void* q, const void* k, const void* v, b2a_dtype in_dtype,
                               int count, void* out, b2a_dtype out_dtype, int nseq = 1);
// safetensors helpers (weights.cu): a byte range of one tensor, and the
// widening of n stored elements of dtype dt to f32 (false: not widenable)
b2a_status st_read_range(const b2a_safetensors* st, const char* name, uint64_t offset, uint64_t length, void* dst);
bool st_widen(const std::string& dt, const void* src, size_t n, float* dst);

// the context's busy flag (one call at a time, src/gpu/model.js:231)
bool ctx_acquire(b2a_ctx* ctx);
void ctx_release(b2a_ctx* ctx);
b2a_status busy_fail(b2a_ctx* ctx);
// frees the context's NCCL gather buffer (b2a_split_kv_decode_nccl)
void nccl_split_release(b2a_ctx* ctx);
// waits for the stream, then reads and clears the device error word
b2a_status stream_sync_check(b2a_ctx* ctx);

}  // namespace b2a
