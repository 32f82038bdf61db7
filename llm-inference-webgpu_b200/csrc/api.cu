// The C ABI of libb2a.so (include/b2a.h): argument validation with the
// reference's error messages, host<->device staging, planning and launches.
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>

#include "b2a_internal.cuh"

// A split-KV exchange (include/b2a.h): one device allocation holding the
// partials [2 parities][world][rows][68] as 64-bit (value, step) words and the
// step / done counters; peer[r] is rank r's allocation as mapped here.
struct b2a_exchange {
  int device = 0;
  int world = 1, rank = 0, batch = 0, layers = 1, heads = 0, kv_heads = 0, rows = 0, groups = 0;
  void* base = nullptr;
  size_t bytes = 0, c_off = 0;
  void* peer[b2a::kMaxWorld] = {};
  bool opened[b2a::kMaxWorld] = {};   // peer[r] came from cudaIpcOpenMemHandle
};

namespace {
thread_local char g_err[1024] = "";
}

namespace b2a {

b2a_status fail(b2a_status s, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return s;
}

b2a_status cuda_fail(cudaError_t e, const char* what) {
  return fail(B2A_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

const char* const kKernelNames[K_NUM_KINDS] = {"attention_simt", "attention_mma", "combine", "rope_append",
                                               "write_at", "grouped_generic", "prefill_tc",
                                               "prefill_pair", "linear_int8", "embed_int8", "rmsnorm",
                                               "swiglu", "argmax", "decode_step"};

namespace {
cudaEvent_t take_event(b2a_ctx* ctx) {
  if (!ctx->event_pool.empty()) {
    cudaEvent_t e = ctx->event_pool.back();
    ctx->event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}
}  // namespace

KernelTimer::KernelTimer(b2a_ctx* ctx, int kind) : ctx_(ctx), kind_(kind) {
  if (!ctx_->timing) {
    done_ = true;
    return;
  }
  start_ = take_event(ctx_);
  if (start_ == nullptr) {
    done_ = true;
    return;
  }
  cudaEventRecord(start_, ctx_->stream);
}

void KernelTimer::stop() {
  if (done_) return;
  done_ = true;
  cudaEvent_t stop = take_event(ctx_);
  if (stop == nullptr) {
    ctx_->event_pool.push_back(start_);
    return;
  }
  cudaEventRecord(stop, ctx_->stream);
  ctx_->timing_recs.push_back({kind_, start_, stop});
}

}  // namespace b2a

using namespace b2a;

namespace {

#define B2A_CUDA(call, what)                      \
  do {                                            \
    cudaError_t e_ = (call);                      \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

// Holds the context for one call: rejects re-entry (src/gpu/model.js:231) and
// makes the context's device current on this thread.
class CallGuard {
 public:
  explicit CallGuard(b2a_ctx* ctx) : ctx_(ctx) {
    int expected = 0;
    ok_ = ctx_ != nullptr && ctx_->busy.compare_exchange_strong(expected, 1);
    if (ok_) cudaSetDevice(ctx_->device);
  }
  ~CallGuard() {
    if (ok_) ctx_->busy.store(0);
  }
  bool ok() const { return ok_; }
  b2a_status busy_status() const {
    if (ctx_ == nullptr) return fail(B2A_EINVAL, "null context");
    return fail(B2A_EBUSY, "a call is already running on this context; wait for it first");
  }

 private:
  b2a_ctx* ctx_;
  bool ok_ = false;
};

b2a_status ensure_buffer(void** buf, size_t* cap, size_t need, const char* what) {
  if (need <= *cap) return B2A_OK;
  if (*buf != nullptr) {
    cudaError_t e = cudaFree(*buf);   // implicitly waits for work that may still use it
    *buf = nullptr;
    *cap = 0;
    if (e != cudaSuccess) return cuda_fail(e, what);
  }
  size_t bytes = need + need / 4 + 4096;
  B2A_CUDA(cudaMalloc(buf, bytes), what);
  *cap = bytes;
  return B2A_OK;
}

bool valid_dtype(int d) { return d == B2A_F32 || d == B2A_F16 || d == B2A_BF16; }

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library needs no link-time libcuda and still loads on a machine without one.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
  }
  return fn;
}

// A pool of `rows` rows of 64 16-bit elements (128 bytes) viewed as a 2D
// tensor; each load is a 64-row box with the 128-byte swizzle the ldmatrix
// reads of the tensor-core decode expect.
bool encode_pool_map(CUtensorMap* map, void* base, uint64_t rows, b2a_dtype dtype) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr || rows >= (1ull << 32)) return false;
  cuuint64_t dims[2] = {64, rows};
  cuuint64_t strides[1] = {128};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype == B2A_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base,
                  dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// A prefill call's rotated f16 queries [rows][heads * 64] as a 2D tensor;
// each load is one head's 128-row query tile, 128-byte swizzled as the
// tensor-core MMAs read it.
bool encode_query_map(CUtensorMap* map, void* q_rot, uint64_t rows, int heads) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr || rows >= (1ull << 32)) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(heads) * 64, rows};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(heads) * 128};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, q_rot, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// A prefill call's 16-bit output [sequences][tokens][heads * 64] as a 3D
// tensor; each store is one head's 128-row tile of one sequence, 128-byte
// swizzled, with the rows past the sequence's tokens clipped.
bool encode_output_map(CUtensorMap* map, void* out, uint64_t nseq, uint64_t tokens, int heads, int out_dtype) {
  EncodeTiledFn fn = encode_tiled();
  if (fn == nullptr || (out_dtype != B2A_F16 && out_dtype != B2A_BF16) || (reinterpret_cast<uintptr_t>(out) & 15) != 0 ||
      tokens >= (1ull << 32) || nseq >= (1ull << 32)) {
    return false;
  }
  const cuuint64_t row = static_cast<cuuint64_t>(heads) * 128;   // bytes
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(heads) * 64, tokens, nseq};
  cuuint64_t strides[2] = {row, row * tokens};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, out_dtype == B2A_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, out,
                  dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Carves device staging for host-pointer calls: each `add` reserves an
// aligned slice of ctx->d_stage.
struct Stage {
  size_t offsets[8];
  size_t sizes[8];
  int n = 0;
  size_t total = 0;
  int add(size_t bytes) {
    offsets[n] = total;
    sizes[n] = bytes;
    total += (bytes + 255) / 256 * 256;
    return n++;
  }
  void* ptr(b2a_ctx* ctx, int i) const { return static_cast<char*>(ctx->d_stage) + offsets[i]; }
};

b2a_status h2d(b2a_ctx* ctx, void* dst, const void* src, size_t bytes) {
  if (bytes == 0) return B2A_OK;
  B2A_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream), "copying inputs to the device");
  return B2A_OK;
}

// The device error word: a kernel whose bounded wait gave up reports it there
// instead of hanging. Host calls read it through pinned host memory with a copy
// enqueued behind their work, so the one stream synchronisation a call makes
// covers its results and the word alike.
b2a_status enqueue_error_read(b2a_ctx* ctx) {
  B2A_CUDA(cudaMemcpyAsync(ctx->h_err, ctx->d_err, sizeof(int32_t), cudaMemcpyDeviceToHost, ctx->stream),
           "reading the device error word");
  return B2A_OK;
}

// Interprets and clears the word read by enqueue_error_read, once the stream is idle.
b2a_status take_error_word(b2a_ctx* ctx) {
  const int32_t err = *ctx->h_err;
  if (err == 0) return B2A_OK;
  *ctx->h_err = 0;
  cudaMemsetAsync(ctx->d_err, 0, sizeof(err), ctx->stream);
  // a kernel that gave up may have left merge counters non-zero
  if (ctx->d_counters) cudaMemsetAsync(ctx->d_counters, 0, ctx->d_counters_bytes, ctx->stream);
  cudaStreamSynchronize(ctx->stream);
  if (err == kErrBadToken) {
    // src/cpu/model.js:203-205
    return fail(B2A_ERANGE, "a token on the device is outside the vocabulary; results of that call are invalid");
  }
  return fail(B2A_ETIMEDOUT, "a device-side wait gave up (error word 0x%x); results of that call are invalid", err);
}

// Waits for the context's stream, then reads and clears the device error word.
b2a_status check_device_error(b2a_ctx* ctx) {
  b2a_status s = enqueue_error_read(ctx);
  if (s != B2A_OK) return s;
  // downloads of asynchronous host-pointer calls run on their own stream
  if (ctx->copy_out) B2A_CUDA(cudaStreamSynchronize(ctx->copy_out), "waiting for the downloads");
  if (ctx->copy_in) B2A_CUDA(cudaStreamSynchronize(ctx->copy_in), "waiting for the uploads");
  B2A_CUDA(cudaStreamSynchronize(ctx->stream), "waiting for the stream");
  return take_error_word(ctx);
}

b2a_status d2h_sync(b2a_ctx* ctx, void* dst, const void* src, size_t bytes) {
  if (bytes) {
    B2A_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream), "copying results to the host");
  }
  b2a_status s = enqueue_error_read(ctx);
  if (s != B2A_OK) return s;
  B2A_CUDA(cudaStreamSynchronize(ctx->stream), "waiting for the results");
  return take_error_word(ctx);
}

b2a_status check_cache_shape(const b2a_kvcache* c, const b2a_rope* rope, int num_heads) {
  if (c == nullptr || rope == nullptr) return fail(B2A_EINVAL, "null cache or rope table");
  if (num_heads <= 0 || num_heads % c->kv_heads != 0) {
    return fail(B2A_EINVAL,
                "num_attention_heads %d is not divisible by num_key_value_heads %d, so the query heads "
                "cannot be grouped evenly over the key/value heads",
                num_heads, c->kv_heads);
  }
  if (rope->head_dim != c->head_dim) {
    return fail(B2A_EINVAL, "rope table head_dim %d differs from the cache's %d", rope->head_dim, c->head_dim);
  }
  if (c->head_dim != 64) return fail(B2A_EINVAL, "cache attention kernels are built for head_dim 64, got %d",
                                     c->head_dim);
  if (num_heads / c->kv_heads > 8) return fail(B2A_EINVAL, "at most 8 query heads per KV head, got %d",
                                               num_heads / c->kv_heads);
  return B2A_OK;
}

// The shortest split-KV chunk, in 64-position tiles: below it the per-chunk
// merge costs more than the parallelism gains.
constexpr int64_t kMinChunkTiles = 4;

AttnParams base_params(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope) {
  AttnParams p{};
  fill_cache_params(p, c);
  p.rope_cos = rope->d_cos;
  p.rope_sin = rope->d_sin;
  p.rope_cos32 = rope->d_cos32;
  p.rope_sin32 = rope->d_sin32;
  p.rope_max = rope->max_positions;
  p.err = ctx->d_err;
  return p;
}

// Splits every query row's keys into chunks, runs the attention kernel into
// the context's scratch, and merges the chunks into `out` (mode 0) or into a
// merged partial (mode 1). max_keys: the longest row's key count.
b2a_status run_split_kv(b2a_ctx* ctx, const b2a_kvcache* c, AttnParams& p, int max_keys, void* out,
                        int out_dtype, int mode) {
  const int64_t rows = static_cast<int64_t>(p.batch) * p.num_layers * p.tokens * p.heads;
  if (rows == 0) return B2A_OK;
  if (c->has_tmaps) {
    p.tmap_k = &c->tmap_k;
    p.tmap_v = &c->tmap_v;
  }
  const bool mma = attn_mma_supported(p);
  // small batches carry their lengths by value: the kernel's work-item lookup
  // then starts without a dependent global load (host and device lengths
  // agree in stream order)
  p.n_len_inline = 0;
  if (p.batch <= kLenInline) {
    for (int b = 0; b < p.batch; b++) p.len_inline[b] = c->len[p.seq_begin + b];
    p.n_len_inline = p.batch;
  }
  p.chunk = 256;
  int64_t items = 0;
  if (mma) {
    // Chunks are whole 64-position tiles. When every (sequence, layer, KV
    // head) group has about the same number of keys and there are fewer
    // groups than resident CTAs (three per SM), split each group into equal
    // chunks that fill the resident CTAs once: one wave of equal items.
    // Otherwise take the longest chunk that still gives every SM several
    // items (about three waves), so the hardware scheduler balances uneven
    // lengths.
    const int64_t slots = 3LL * ctx->sm_count;
    const int64_t groups = static_cast<int64_t>(p.batch) * p.num_layers * p.kv_heads;
    int min_nk = INT32_MAX, max_nk = 0;
    for (int b = 0; b < p.batch; b++) {
      const int nk = c->len[p.seq_begin + b] + p.horizon_extra;
      min_nk = std::min(min_nk, nk);
      max_nk = std::max(max_nk, nk);
    }
    const int64_t per_group = groups > 0 ? slots / groups : 0;
    if (mode == 2) {
      // the exchange waits inside the kernel: every CTA must be resident at
      // once, so one wave with at most kMaxFusedChunks chunks per group
      if (per_group < 1) {
        return fail(B2A_EINVAL, "%lld (sequence, KV head) groups exceed the %lld CTAs resident at once",
                    static_cast<long long>(groups), static_cast<long long>(slots));
      }
      const int64_t tiles = (std::max(max_nk, 1) + 63) / 64;
      const int64_t n = std::min<int64_t>(per_group, attn_mma_max_fused_chunks());
      p.chunk = static_cast<int>(64 * std::max<int64_t>(kMinChunkTiles, (tiles + n - 1) / n));
      items = attn_mma_items(p, c->len.data());
    } else if (per_group >= 2 && max_nk > 0 &&
               static_cast<int64_t>(min_nk) * 8 >= static_cast<int64_t>(max_nk) * 7) {
      const int64_t tiles = (max_nk + 63) / 64;
      p.chunk = static_cast<int>(64 * std::max<int64_t>(kMinChunkTiles, (tiles + per_group - 1) / per_group));
      items = attn_mma_items(p, c->len.data());
    } else {
      // about two waves of the resident CTAs over all the key tiles, in chunks
      // of 4..64 tiles: short work keeps whole groups in one chunk (no merge),
      // a long multi-layer batch gets whole 4096-position chunks
      int64_t total_tiles = 0;
      for (int b = 0; b < p.batch; b++) {
        total_tiles += (static_cast<int64_t>(c->len[p.seq_begin + b]) + p.horizon_extra + 63) / 64;
      }
      total_tiles *= static_cast<int64_t>(p.num_layers) * p.kv_heads;
      const int64_t per_item = (total_tiles + 2 * slots - 1) / (2 * slots);
      p.chunk = static_cast<int>(64 * std::min<int64_t>(64, std::max<int64_t>(kMinChunkTiles, per_item)));
      items = attn_mma_items(p, c->len.data());
    }
  }
  p.nchunks = max_keys > 0 ? (max_keys + p.chunk - 1) / p.chunk : 1;
  const size_t need = static_cast<size_t>(rows) * p.nchunks * (p.head_dim + 4) * sizeof(float);
  b2a_status s = ensure_buffer(&ctx->d_scratch, &ctx->d_scratch_bytes, need, "allocating split-KV scratch");
  if (s != B2A_OK) return s;
  p.partial = static_cast<float*>(ctx->d_scratch);
  // the tensor-core kernel merges its own chunks when they are few: one CTA
  // walking many chunks would be a long tail, which the parallel combine avoids
  const bool fused = mma && p.nchunks <= attn_mma_max_fused_chunks();
  if (mode == 2 && !fused) return fail(B2A_EINVAL, "the split exchange needs an f16 or bf16 cache");
  if (fused) {
    const size_t cbytes = static_cast<size_t>(p.batch) * p.num_layers * p.kv_heads * sizeof(int32_t);
    if (cbytes > ctx->d_counters_bytes) {
      void* buf = ctx->d_counters;
      size_t cap = ctx->d_counters_bytes;
      if ((s = ensure_buffer(&buf, &cap, cbytes, "allocating merge counters")) != B2A_OK) return s;
      ctx->d_counters = static_cast<int32_t*>(buf);
      ctx->d_counters_bytes = cap;
      B2A_CUDA(cudaMemsetAsync(ctx->d_counters, 0, cap, ctx->stream), "clearing merge counters");
    }
    p.fuse_out = out;
    p.fuse_dtype = out_dtype;
    p.fuse_mode = mode;
    p.counters = ctx->d_counters;
  }
  cudaError_t e;
  {
    KernelTimer kt(ctx, mma ? K_ATTN_MMA : K_ATTN_SIMT);
    e = mma ? launch_attn_mma(p, items, ctx->stream) : launch_attn_simt(p, ctx->stream);
  }
  if (e != cudaSuccess) return cuda_fail(e, "launching the attention kernel");
  if (fused) return B2A_OK;
  CombineParams cp{};
  cp.partial = p.partial;
  cp.rows = rows;
  cp.nchunks = p.nchunks;
  cp.head_dim = p.head_dim;
  cp.part_stride_rows = 0;
  cp.out = out;
  cp.out_dtype = out_dtype;
  cp.mode = mode;
  cp.len = p.len;
  cp.seq_begin = p.seq_begin;
  cp.chunk = p.chunk;
  cp.extra = p.horizon_extra;
  cp.tokens = p.tokens;
  cp.heads = p.heads;
  cp.num_layers = p.num_layers;
  {
    KernelTimer kt(ctx, K_COMBINE);
    e = launch_combine(cp, ctx->stream);
  }
  if (e != cudaSuccess) return cuda_fail(e, "launching the split-KV combine");
  return B2A_OK;
}

// Host-pointer decode, pipelined over groups of sequences: each group's upload
// (copy_in stream), attention kernels (the context's stream) and download
// (copy_out stream) overlap those of its neighbours, so the PCIe transfers hide
// behind the HBM-bound kernels. p carries the device staging pointers of the
// whole batch; q_seq / kv_seq / out_seq are the bytes per sequence.
b2a_status decode_host_pipelined(b2a_ctx* ctx, const b2a_kvcache* c, const AttnParams& p, const void* hq,
                                 const void* hk, const void* hv, void* hout, void* dout, int out_dtype, size_t q_seq,
                                 size_t kv_seq, size_t out_seq, int async_slot) {
  const int batch = p.batch;
  const int layers = p.num_layers;
  const size_t seq_bytes = q_seq + (hk ? 2 * kv_seq : 0) + out_seq;
  // Several layers: groups of whole layers for every sequence, so each group's
  // kernel sees the whole batch (balanced, full-length chunks) and its copies
  // are strided 2D copies into dense per-group staging. One layer: groups of
  // sequences. ~3 MiB of transfers per group and at most 3 groups either way:
  // measured on config 3 (9 MB per call), 1 / 3 / 6 / 8 layer groups took
  // 0.54 / 0.44 / 0.44 / 0.49 ms per call; more groups add per-group launch
  // and copy overhead (and, for sequence groups, shorter chunks and tails)
  // faster than they hide copies.
  const bool by_layer = layers >= 2;
  int groups;
  if (by_layer) {
    groups = static_cast<int>(std::min<size_t>(3, std::max<size_t>(1, batch * seq_bytes / (3u << 20))));
    if (groups > layers) groups = layers;
  } else {
    groups = static_cast<int>(std::min<size_t>(3, std::max<size_t>(1, batch * seq_bytes / (3u << 20))));
    if (groups > batch) groups = batch;
  }
  if (ctx->copy_in == nullptr) {
    B2A_CUDA(cudaStreamCreateWithFlags(&ctx->copy_in, cudaStreamNonBlocking), "creating the upload stream");
  }
  if (ctx->copy_out == nullptr) {
    B2A_CUDA(cudaStreamCreateWithFlags(&ctx->copy_out, cudaStreamNonBlocking), "creating the download stream");
  }
  while (ctx->pipe_events.size() < static_cast<size_t>(2 * groups + 1)) {
    cudaEvent_t e;
    B2A_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "creating pipeline events");
    ctx->pipe_events.push_back(e);
  }
  if (async_slot < 0) {
    // uploads wait for earlier work on the context's stream (it may still read the staging buffer)
    cudaEvent_t start = ctx->pipe_events[2 * groups];
    B2A_CUDA(cudaEventRecord(start, ctx->stream), "ordering the upload");
    B2A_CUDA(cudaStreamWaitEvent(ctx->copy_in, start, 0), "ordering the upload");
  } else if (ctx->async_used[async_slot]) {
    // this staging slot's previous call has downloaded its last result (and
    // so run its last kernel): the uploads may overwrite it; the other slot's
    // call may still be running, which is what lets consecutive calls overlap
    B2A_CUDA(cudaStreamWaitEvent(ctx->copy_in, ctx->async_free[async_slot], 0), "ordering the upload");
  }
  const char* src_q = static_cast<const char*>(hq);
  char* dst_q = static_cast<char*>(const_cast<void*>(p.q));
  if (by_layer) {
    // per layer and sequence: q, new k/v and out bytes
    const size_t ql = q_seq / layers, kvl = kv_seq / layers, ol = out_seq / layers;
    char* dst_k = static_cast<char*>(const_cast<void*>(p.k_new));
    char* dst_v = static_cast<char*>(const_cast<void*>(p.v_new));
    int max_keys = 0;
    for (int b = p.seq_begin; b < p.seq_begin + batch; b++) max_keys = std::max(max_keys, c->len[b] + p.horizon_extra);
    // issued group by group (upload, kernel, download), so the first kernel
    // is enqueued after one group's copies rather than after all of them
    for (int gi = 0; gi < groups; gi++) {
      const int l0 = layers * gi / groups, l1 = layers * (gi + 1) / groups, n = l1 - l0;
      // host [batch][layers][...] rows -> dense staging [batch][n][...] at batch * l0 layer slots
      B2A_CUDA(cudaMemcpy2DAsync(dst_q + batch * l0 * ql, n * ql, src_q + l0 * ql, q_seq, n * ql, batch,
                                 cudaMemcpyHostToDevice, ctx->copy_in),
               "copying q to the device");
      if (hk) {
        B2A_CUDA(cudaMemcpy2DAsync(dst_k + batch * l0 * kvl, n * kvl, static_cast<const char*>(hk) + l0 * kvl, kv_seq,
                                   n * kvl, batch, cudaMemcpyHostToDevice, ctx->copy_in),
                 "copying new keys to the device");
        B2A_CUDA(cudaMemcpy2DAsync(dst_v + batch * l0 * kvl, n * kvl, static_cast<const char*>(hv) + l0 * kvl, kv_seq,
                                   n * kvl, batch, cudaMemcpyHostToDevice, ctx->copy_in),
                 "copying new values to the device");
      }
      B2A_CUDA(cudaEventRecord(ctx->pipe_events[2 * gi], ctx->copy_in), "recording an upload");
      B2A_CUDA(cudaStreamWaitEvent(ctx->stream, ctx->pipe_events[2 * gi], 0), "waiting for an upload");
      AttnParams pg = p;
      pg.layer_begin = p.layer_begin + l0;
      pg.num_layers = n;
      pg.q = dst_q + batch * l0 * ql;
      if (hk) {
        pg.k_new = dst_k + batch * l0 * kvl;
        pg.v_new = dst_v + batch * l0 * kvl;
      }
      char* gout = static_cast<char*>(dout) + batch * l0 * ol;
      b2a_status s = run_split_kv(ctx, c, pg, max_keys, gout, out_dtype, 0);
      if (s != B2A_OK) return s;
      B2A_CUDA(cudaEventRecord(ctx->pipe_events[2 * gi + 1], ctx->stream), "recording a group");
      B2A_CUDA(cudaStreamWaitEvent(ctx->copy_out, ctx->pipe_events[2 * gi + 1], 0), "ordering a download");
      B2A_CUDA(cudaMemcpy2DAsync(static_cast<char*>(hout) + l0 * ol, out_seq, gout, n * ol, n * ol, batch,
                                 cudaMemcpyDeviceToHost, ctx->copy_out),
               "copying results to the host");
    }
    if (async_slot >= 0) {
      B2A_CUDA(cudaEventRecord(ctx->async_free[async_slot], ctx->copy_out), "recording the slot's last download");
      ctx->async_used[async_slot] = true;
      return B2A_OK;
    }
    b2a_status es = enqueue_error_read(ctx);
    if (es != B2A_OK) return es;
    B2A_CUDA(cudaStreamSynchronize(ctx->copy_out), "waiting for the results");
    B2A_CUDA(cudaStreamSynchronize(ctx->stream), "waiting for the kernels");
    return take_error_word(ctx);
  }
  for (int gi = 0; gi < groups; gi++) {
    const int b0 = static_cast<int>(static_cast<int64_t>(batch) * gi / groups);
    const int b1 = static_cast<int>(static_cast<int64_t>(batch) * (gi + 1) / groups);
    const int n = b1 - b0;
    if (n == 0) continue;
    B2A_CUDA(cudaMemcpyAsync(dst_q + b0 * q_seq, src_q + b0 * q_seq, n * q_seq, cudaMemcpyHostToDevice,
                             ctx->copy_in),
             "copying q to the device");
    if (hk) {
      B2A_CUDA(cudaMemcpyAsync(static_cast<char*>(const_cast<void*>(p.k_new)) + b0 * kv_seq,
                               static_cast<const char*>(hk) + b0 * kv_seq, n * kv_seq, cudaMemcpyHostToDevice,
                               ctx->copy_in),
               "copying new keys to the device");
      B2A_CUDA(cudaMemcpyAsync(static_cast<char*>(const_cast<void*>(p.v_new)) + b0 * kv_seq,
                               static_cast<const char*>(hv) + b0 * kv_seq, n * kv_seq, cudaMemcpyHostToDevice,
                               ctx->copy_in),
               "copying new values to the device");
    }
    B2A_CUDA(cudaEventRecord(ctx->pipe_events[2 * gi], ctx->copy_in), "recording an upload");
  }
  for (int gi = 0; gi < groups; gi++) {
    const int b0 = static_cast<int>(static_cast<int64_t>(batch) * gi / groups);
    const int b1 = static_cast<int>(static_cast<int64_t>(batch) * (gi + 1) / groups);
    const int n = b1 - b0;
    if (n == 0) continue;
    B2A_CUDA(cudaStreamWaitEvent(ctx->stream, ctx->pipe_events[2 * gi], 0), "waiting for an upload");
    AttnParams pg = p;
    pg.seq_begin = p.seq_begin + b0;
    pg.batch = n;
    pg.q = dst_q + b0 * q_seq;
    if (hk) {
      pg.k_new = static_cast<const char*>(p.k_new) + b0 * kv_seq;
      pg.v_new = static_cast<const char*>(p.v_new) + b0 * kv_seq;
    }
    int max_keys = 0;
    for (int b = pg.seq_begin; b < pg.seq_begin + n; b++) max_keys = std::max(max_keys, c->len[b] + p.horizon_extra);
    b2a_status s = run_split_kv(ctx, c, pg, max_keys, static_cast<char*>(dout) + b0 * out_seq, out_dtype, 0);
    if (s != B2A_OK) return s;
    B2A_CUDA(cudaEventRecord(ctx->pipe_events[2 * gi + 1], ctx->stream), "recording a group");
    B2A_CUDA(cudaStreamWaitEvent(ctx->copy_out, ctx->pipe_events[2 * gi + 1], 0), "ordering a download");
    B2A_CUDA(cudaMemcpyAsync(static_cast<char*>(hout) + b0 * out_seq, static_cast<char*>(dout) + b0 * out_seq,
                             n * out_seq, cudaMemcpyDeviceToHost, ctx->copy_out),
             "copying results to the host");
  }
  if (async_slot >= 0) {
    B2A_CUDA(cudaEventRecord(ctx->async_free[async_slot], ctx->copy_out), "recording the slot's last download");
    ctx->async_used[async_slot] = true;
    return B2A_OK;
  }
  b2a_status es = enqueue_error_read(ctx);
  if (es != B2A_OK) return es;
  B2A_CUDA(cudaStreamSynchronize(ctx->copy_out), "waiting for the results");
  B2A_CUDA(cudaStreamSynchronize(ctx->stream), "waiting for the kernels");
  return take_error_word(ctx);
}


// A new token's attention over the positions this cache holds (split-KV
// decode): ex == nullptr writes the partials [batch][heads][D+4] (fuse mode 1);
// otherwise the kernel exchanges them with the other ranks and writes the
// combined output in out_dtype (fuse mode 2).
b2a_status decode_positions(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope, int layer, int num_layers,
                            int num_heads, const void* q, const void* k_new, const void* v_new, b2a_dtype in_dtype,
                            const int32_t* q_positions, b2a_exchange* ex, void* out, b2a_dtype out_dtype, int flags) {
  b2a_status s = check_cache_shape(c, rope, num_heads);
  if (s != B2A_OK) return s;
  if (q == nullptr || out == nullptr || q_positions == nullptr) return fail(B2A_EINVAL, "null argument");
  if ((k_new == nullptr) != (v_new == nullptr)) return fail(B2A_EINVAL, "give both new keys and values, or neither");
  if (!valid_dtype(in_dtype)) return fail(B2A_EINVAL, "unknown dtype");
  if (layer < 0 || num_layers < 1 || layer + num_layers > c->layers) {
    return fail(B2A_EINVAL, "layers [%d, %d) outside the cache's %d", layer, layer + num_layers, c->layers);
  }
  const int extra = k_new ? 1 : 0;
  int max_keys = 0;
  for (int b = 0; b < c->batch; b++) {
    if (c->len[b] + extra > c->capacity) {
      return fail(B2A_ERANGE, "cache holds %d of %d positions; cannot add %d more", c->len[b], c->capacity, extra);
    }
    if (c->len[b] + extra > max_keys) max_keys = c->len[b] + extra;
  }
  if (flags == B2A_HOST) {
    for (int b = 0; b < c->batch; b++) {
      if (q_positions[b] < 0 || q_positions[b] >= rope->max_positions) {
        return fail(B2A_ERANGE, "position %d exceeds the %d-entry rope table", q_positions[b] + 1, rope->max_positions);
      }
    }
  }
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  if ((s = cache_reserve_all(c, extra)) != B2A_OK) return s;
  AttnParams p = base_params(ctx, c, rope);
  p.seq_begin = 0;
  p.batch = c->batch;
  p.num_layers = num_layers;
  p.layer_begin = layer;
  p.tokens = 1;
  p.heads = num_heads;
  p.group = num_heads / c->kv_heads;
  p.in_dtype = static_cast<int>(in_dtype);
  p.q = q;
  p.k_new = k_new;
  p.v_new = v_new;
  p.q_pos = q_positions;
  p.horizon_extra = extra;
  const int mode = ex ? 2 : 1;
  const b2a_dtype odt = ex ? out_dtype : B2A_F32;
  if (ex) {
    for (int r = 0; r < ex->world; r++) {
      p.x_peer[r] = static_cast<uint64_t*>(ex->peer[r]);
    }
    p.x_local = static_cast<const uint64_t*>(ex->base);
    p.x_epoch = reinterpret_cast<int32_t*>(static_cast<char*>(ex->base) + ex->c_off);
    p.x_done = p.x_epoch + 1;
    p.x_world = ex->world;
    p.x_rank = ex->rank;
    p.x_rows = ex->rows;
  }
  const size_t ies = dtype_size(in_dtype);
  const size_t rows_bl = static_cast<size_t>(c->batch) * num_layers;   // (sequence, layer) pairs
  const size_t q_bytes = rows_bl * num_heads * c->head_dim * ies;
  const size_t kv_bytes = rows_bl * c->kv_heads * c->head_dim * ies;
  const size_t out_bytes = rows_bl * num_heads *
                           (ex ? c->head_dim * dtype_size(out_dtype) : (c->head_dim + 4) * sizeof(float));
  void* dout = out;
  if (flags == B2A_HOST) {
    Stage st;
    int iq = st.add(q_bytes), ik = st.add(k_new ? kv_bytes : 0), iv = st.add(k_new ? kv_bytes : 0),
        io = st.add(out_bytes), ipos = st.add(sizeof(int32_t) * c->batch);
    if ((s = ensure_buffer(&ctx->d_stage, &ctx->d_stage_bytes, st.total, "allocating staging")) != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, iq), q, q_bytes)) != B2A_OK) return s;
    p.q = st.ptr(ctx, iq);
    if (k_new) {
      if ((s = h2d(ctx, st.ptr(ctx, ik), k_new, kv_bytes)) != B2A_OK) return s;
      if ((s = h2d(ctx, st.ptr(ctx, iv), v_new, kv_bytes)) != B2A_OK) return s;
      p.k_new = st.ptr(ctx, ik);
      p.v_new = st.ptr(ctx, iv);
    }
    if ((s = h2d(ctx, st.ptr(ctx, ipos), q_positions, sizeof(int32_t) * c->batch)) != B2A_OK) return s;
    p.q_pos = static_cast<const int32_t*>(st.ptr(ctx, ipos));
    dout = st.ptr(ctx, io);
  }
  if ((s = run_split_kv(ctx, c, p, max_keys, dout, static_cast<int>(odt), mode)) != B2A_OK) return s;
  if (flags == B2A_HOST) return d2h_sync(ctx, out, dout, out_bytes);
  return B2A_OK;
}


// Shared body of b2a_linear_int8 / b2a_qkv_int8: validation, staging of host
// pointers, launch. seg_end lists the cumulative rows of each output.
b2a_status linear_int8(b2a_ctx* ctx, const int8_t* codes, const void* scales, b2a_dtype scale_dtype, const void* bias,
                       b2a_dtype bias_dtype, const void* x, b2a_dtype x_dtype, int rows, int cols, int tokens,
                       const void* residual, void* const* outs, const int* seg_end, int nseg, b2a_dtype out_dtype,
                       int flags) {
  if (ctx == nullptr || codes == nullptr || scales == nullptr || x == nullptr) return fail(B2A_EINVAL, "null argument");
  for (int s = 0; s < nseg; s++)
    if (outs[s] == nullptr) return fail(B2A_EINVAL, "null argument");
  if (!valid_dtype(scale_dtype) || !valid_dtype(bias_dtype) || !valid_dtype(x_dtype) || !valid_dtype(out_dtype)) {
    return fail(B2A_EINVAL, "unknown dtype");
  }
  if (rows < 1 || cols < 16 || cols % 16 != 0 || tokens < 0) {
    return fail(B2A_EINVAL, "linear shape: rows %d, cols %d (a positive multiple of 16), tokens %d", rows, cols, tokens);
  }
  if (tokens == 0) return B2A_OK;
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  const size_t w_bytes = static_cast<size_t>(rows) * cols;
  const size_t sc_bytes = static_cast<size_t>(rows) * dtype_size(scale_dtype);
  const size_t b_bytes = bias ? static_cast<size_t>(rows) * dtype_size(bias_dtype) : 0;
  const size_t x_bytes = static_cast<size_t>(tokens) * cols * dtype_size(x_dtype);
  LinearParams p{};
  p.w = codes;
  p.scale = scales;
  p.scale_dtype = static_cast<int>(scale_dtype);
  p.bias = bias;
  p.bias_dtype = static_cast<int>(bias_dtype);
  p.x = x;
  p.x_dtype = static_cast<int>(x_dtype);
  p.rows = rows;
  p.cols = cols;
  p.tokens = tokens;
  p.nseg = nseg;
  p.out_dtype = static_cast<int>(out_dtype);
  p.residual = residual;
  size_t out_bytes[3] = {0, 0, 0};
  for (int s = 0; s < nseg; s++) {
    p.seg_end[s] = seg_end[s];
    p.out[s] = outs[s];
    out_bytes[s] = static_cast<size_t>(tokens) * (seg_end[s] - (s ? seg_end[s - 1] : 0)) * dtype_size(out_dtype);
  }
  b2a_status st;
  if (flags == B2A_HOST) {
    Stage sg;
    int iw = sg.add(w_bytes), is = sg.add(sc_bytes), ib = sg.add(b_bytes), ix = sg.add(x_bytes),
        ir = sg.add(residual ? out_bytes[0] : 0);
    int io[3] = {sg.add(out_bytes[0]), sg.add(out_bytes[1]), sg.add(out_bytes[2])};
    if ((st = ensure_buffer(&ctx->d_stage, &ctx->d_stage_bytes, sg.total, "allocating staging")) != B2A_OK) return st;
    if ((st = h2d(ctx, sg.ptr(ctx, iw), codes, w_bytes)) != B2A_OK) return st;
    if ((st = h2d(ctx, sg.ptr(ctx, is), scales, sc_bytes)) != B2A_OK) return st;
    if (bias && (st = h2d(ctx, sg.ptr(ctx, ib), bias, b_bytes)) != B2A_OK) return st;
    if ((st = h2d(ctx, sg.ptr(ctx, ix), x, x_bytes)) != B2A_OK) return st;
    if (residual && (st = h2d(ctx, sg.ptr(ctx, ir), residual, out_bytes[0])) != B2A_OK) return st;
    p.w = static_cast<const int8_t*>(sg.ptr(ctx, iw));
    p.scale = sg.ptr(ctx, is);
    p.bias = bias ? sg.ptr(ctx, ib) : nullptr;
    p.x = sg.ptr(ctx, ix);
    p.residual = residual ? sg.ptr(ctx, ir) : nullptr;
    for (int s = 0; s < nseg; s++) p.out[s] = sg.ptr(ctx, io[s]);
  } else if ((reinterpret_cast<uintptr_t>(codes) & 15) != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0) {
    return fail(B2A_EINVAL, "device codes and activations must start on a 16-byte boundary");
  }
  cudaError_t e;
  {
    KernelTimer kt(ctx, K_LINEAR);
    e = launch_linear_int8(p, ctx->stream);
  }
  if (e != cudaSuccess) return cuda_fail(e, "launching the int8 projection");
  if (flags == B2A_HOST) {
    for (int s = 0; s < nseg; s++) {
      B2A_CUDA(cudaMemcpyAsync(outs[s], p.out[s], out_bytes[s], cudaMemcpyDeviceToHost, ctx->stream),
               "copying results to the host");
    }
    return d2h_sync(ctx, nullptr, nullptr, 0);
  }
  return B2A_OK;
}

}  // namespace

namespace b2a {
bool ctx_acquire(b2a_ctx* ctx) {
  int expected = 0;
  if (ctx == nullptr || !ctx->busy.compare_exchange_strong(expected, 1)) return false;
  cudaSetDevice(ctx->device);
  return true;
}
void ctx_release(b2a_ctx* ctx) { ctx->busy.store(0); }
b2a_status busy_fail(b2a_ctx* ctx) {
  if (ctx == nullptr) return fail(B2A_EINVAL, "null context");
  return fail(B2A_EBUSY, "a call is already running on this context; wait for it first");
}
b2a_status stream_sync_check(b2a_ctx* ctx) { return d2h_sync(ctx, nullptr, nullptr, 0); }
}  // namespace b2a

extern "C" {

const char* b2a_last_error(void) { return g_err; }

const char* b2a_status_name(b2a_status s) {
  switch (s) {
    case B2A_OK: return "B2A_OK";
    case B2A_EINVAL: return "B2A_EINVAL";
    case B2A_ERANGE: return "B2A_ERANGE";
    case B2A_EBUSY: return "B2A_EBUSY";
    case B2A_ECUDA: return "B2A_ECUDA";
    case B2A_ENCCL: return "B2A_ENCCL";
    case B2A_ETIMEDOUT: return "B2A_ETIMEDOUT";
    case B2A_ENODEV: return "B2A_ENODEV";
  }
  return "B2A_UNKNOWN";
}

int b2a_abi_version(void) { return B2A_ABI_VERSION; }

// ---------------------------------------------------------------- context --

b2a_status b2a_init(int device, b2a_ctx** out) {
  if (out == nullptr) return fail(B2A_EINVAL, "null output pointer");
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    return fail(B2A_ENODEV, "no CUDA device available (%s)", e != cudaSuccess ? cudaGetErrorString(e) : "0 devices");
  }
  if (device < 0 || device >= count) return fail(B2A_ENODEV, "device %d out of range (%d devices)", device, count);
  B2A_CUDA(cudaSetDevice(device), "selecting the device");
  cudaDeviceProp prop;
  B2A_CUDA(cudaGetDeviceProperties(&prop, device), "querying the device");
  if (prop.major != 10) {
    return fail(B2A_ENODEV, "device %d is sm_%d%d; this library is built for sm_100a (B200)", device, prop.major,
                prop.minor);
  }
  b2a_ctx* ctx = new (std::nothrow) b2a_ctx();
  if (ctx == nullptr) return fail(B2A_EINVAL, "out of host memory");
  ctx->device = device;
  ctx->sm_count = prop.multiProcessorCount;
  e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete ctx;
    return cuda_fail(e, "creating the stream");
  }
  ctx->stream = ctx->own_stream;
  e = cudaMalloc(&ctx->d_err, 64);
  if (e == cudaSuccess) e = cudaMemset(ctx->d_err, 0, 64);
  if (e == cudaSuccess) e = cudaHostAlloc(reinterpret_cast<void**>(&ctx->h_err), 64, cudaHostAllocDefault);
  if (e != cudaSuccess) {
    if (ctx->d_err) cudaFree(ctx->d_err);
    cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return cuda_fail(e, "allocating the error word");
  }
  *ctx->h_err = 0;
  // the no-alloc decode's scratch array and kernels become resident now, while
  // the host can still allocate (the runtime would otherwise load them lazily
  // at that decode's first call)
  b2a_status s = noalloc_prepare(device);
  if (s != B2A_OK) {
    cudaFreeHost(ctx->h_err);
    cudaFree(ctx->d_err);
    cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return s;
  }
  *out = ctx;
  return B2A_OK;
}

b2a_status b2a_destroy(b2a_ctx* ctx) {
  if (ctx == nullptr) return B2A_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->d_stage) cudaFree(ctx->d_stage);
  if (ctx->copy_out) cudaStreamSynchronize(ctx->copy_out);
  for (int i = 0; i < 2; i++) {
    if (ctx->d_async[i]) cudaFree(ctx->d_async[i]);
    if (ctx->async_free[i]) cudaEventDestroy(ctx->async_free[i]);
  }
  if (ctx->d_scratch) cudaFree(ctx->d_scratch);
  if (ctx->d_qrot) cudaFree(ctx->d_qrot);
  nccl_split_release(ctx);
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->h_err) cudaFreeHost(ctx->h_err);
  if (ctx->d_positions) cudaFree(ctx->d_positions);
  if (ctx->d_counters) cudaFree(ctx->d_counters);
  for (auto& r : ctx->timing_recs) {
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  for (auto ev : ctx->event_pool) cudaEventDestroy(ev);
  for (auto ev : ctx->pipe_events) cudaEventDestroy(ev);
  if (ctx->copy_in) cudaStreamDestroy(ctx->copy_in);
  if (ctx->copy_out) cudaStreamDestroy(ctx->copy_out);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
  return B2A_OK;
}

b2a_status b2a_set_stream(b2a_ctx* ctx, void* cuda_stream) {
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  ctx->stream = cuda_stream ? static_cast<cudaStream_t>(cuda_stream) : ctx->own_stream;
  return B2A_OK;
}

b2a_status b2a_synchronize(b2a_ctx* ctx) {
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  return check_device_error(ctx);
}

b2a_status b2a_timing_enable(b2a_ctx* ctx, int enable) {
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  ctx->timing = enable != 0;
  return B2A_OK;
}

b2a_status b2a_timing_read(b2a_ctx* ctx, b2a_kernel_time* out, int max_entries, int* n_entries) {
  if (out == nullptr || n_entries == nullptr || max_entries < 0) return fail(B2A_EINVAL, "null argument");
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  B2A_CUDA(cudaStreamSynchronize(ctx->stream), "waiting for timed kernels");
  int launches[K_NUM_KINDS] = {0};
  double ms[K_NUM_KINDS] = {0};
  for (auto& r : ctx->timing_recs) {
    float t = 0.f;
    if (cudaEventElapsedTime(&t, r.start, r.stop) == cudaSuccess) {
      launches[r.kind]++;
      ms[r.kind] += t;
    }
    ctx->event_pool.push_back(r.start);
    ctx->event_pool.push_back(r.stop);
  }
  ctx->timing_recs.clear();
  int n = 0;
  for (int k = 0; k < K_NUM_KINDS && n < max_entries; k++) {
    if (launches[k] == 0) continue;
    snprintf(out[n].name, sizeof(out[n].name), "%s", kKernelNames[k]);
    out[n].launches = launches[k];
    out[n].total_ms = ms[k];
    n++;
  }
  *n_entries = n;
  return B2A_OK;
}

// ------------------------------------------------------------ host helpers --

int b2a_kv_head_for(int query_head, int num_heads, int num_kv_heads) {
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0) return -1;
  if (query_head < 0 || query_head >= num_heads) return -1;
  return query_head / (num_heads / num_kv_heads);
}

b2a_status b2a_rope_frequencies(int head_dim, double theta, double* inv_freq) {
  if (head_dim <= 0 || head_dim % 2 != 0 || inv_freq == nullptr) {
    return fail(B2A_EINVAL, "head_dim must be a positive even number, got %d", head_dim);
  }
  const int half = head_dim >> 1;
  for (int j = 0; j < half; j++) inv_freq[j] = std::pow(theta, static_cast<double>(-2 * j) / head_dim);
  return B2A_OK;
}

b2a_status b2a_rope_tables(int head_dim, double theta, int positions, float* cos_out, float* sin_out) {
  if (positions < 0 || cos_out == nullptr || sin_out == nullptr) return fail(B2A_EINVAL, "bad rope table arguments");
  double inv[512];
  if (head_dim > 1024) return fail(B2A_EINVAL, "head_dim %d too large", head_dim);
  b2a_status s = b2a_rope_frequencies(head_dim, theta, inv);
  if (s != B2A_OK) return s;
  const int half = head_dim >> 1;
  for (int p = 0; p < positions; p++) {
    for (int j = 0; j < half; j++) {
      const double angle = static_cast<double>(p) * inv[j];
      cos_out[static_cast<size_t>(p) * half + j] = static_cast<float>(std::cos(angle));
      sin_out[static_cast<size_t>(p) * half + j] = static_cast<float>(std::sin(angle));
    }
  }
  return B2A_OK;
}

// -------------------------------------------------------------- rope table --

b2a_status b2a_rope_create(b2a_ctx* ctx, int head_dim, double theta, int max_positions, b2a_rope** out) {
  if (out == nullptr) return fail(B2A_EINVAL, "null output pointer");
  *out = nullptr;
  if (head_dim <= 0 || head_dim % 2 != 0 || head_dim > 1024) {
    return fail(B2A_EINVAL, "head_dim must be a positive even number <= 1024, got %d", head_dim);
  }
  if (max_positions < 1) return fail(B2A_ERANGE, "rope table needs at least one position, got %d", max_positions);
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  const int half = head_dim >> 1;
  double inv[512];
  b2a_rope_frequencies(head_dim, theta, inv);
  const size_t n = static_cast<size_t>(max_positions) * half;
  // one pinned block: cos f64, sin f64, cos f32, sin f32
  void* host = nullptr;
  B2A_CUDA(cudaMallocHost(&host, n * 2 * (sizeof(double) + sizeof(float))), "allocating the host rope table");
  double* hc = static_cast<double*>(host);
  double* hs = hc + n;
  float* hc32 = reinterpret_cast<float*>(hs + n);
  float* hs32 = hc32 + n;
  // The angle ropeInPlace evaluates (src/core/ops.js:150-152), in f64.
  for (int p = 0; p < max_positions; p++) {
    for (int j = 0; j < half; j++) {
      const size_t i = static_cast<size_t>(p) * half + j;
      const double angle = static_cast<double>(p) * inv[j];
      hc[i] = std::cos(angle);
      hs[i] = std::sin(angle);
      hc32[i] = static_cast<float>(hc[i]);
      hs32[i] = static_cast<float>(hs[i]);
    }
  }
  b2a_rope* r = new (std::nothrow) b2a_rope();
  if (r == nullptr) {
    cudaFreeHost(host);
    return fail(B2A_ECUDA, "out of host memory for the rope table");
  }
  r->ctx = ctx;
  r->device = ctx->device;
  r->head_dim = head_dim;
  r->theta = theta;
  r->max_positions = max_positions;
  cudaError_t e = cudaMalloc(&r->d_cos, n * sizeof(double));
  if (e == cudaSuccess) e = cudaMalloc(&r->d_sin, n * sizeof(double));
  if (e == cudaSuccess) e = cudaMalloc(&r->d_cos32, n * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&r->d_sin32, n * sizeof(float));
  if (e == cudaSuccess) e = cudaMemcpyAsync(r->d_cos, hc, n * sizeof(double), cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(r->d_sin, hs, n * sizeof(double), cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(r->d_cos32, hc32, n * sizeof(float), cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(r->d_sin32, hs32, n * sizeof(float), cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  cudaFreeHost(host);
  if (e != cudaSuccess) {
    cudaFree(r->d_cos);
    cudaFree(r->d_sin);
    cudaFree(r->d_cos32);
    cudaFree(r->d_sin32);
    delete r;
    return cuda_fail(e, "uploading the rope table");
  }
  *out = r;
  return B2A_OK;
}

// Destruction touches only the object's own device memory (cudaFree waits for
// work still using it), so it is safe after the context is gone.
b2a_status b2a_rope_destroy(b2a_rope* rope) {
  if (rope == nullptr) return B2A_OK;
  cudaSetDevice(rope->device);
  cudaFree(rope->d_cos);
  cudaFree(rope->d_sin);
  cudaFree(rope->d_cos32);
  cudaFree(rope->d_sin32);
  delete rope;
  return B2A_OK;
}

// ---------------------------------------------------------------- KV cache --

}  // extern "C"

namespace b2a {
namespace {

// A contiguous cache (page_size 0: batch blocks of capacity positions) or a
// paged one (num_pages + 1 pages of page_size positions, the last one the
// scratch page that unmapped page-table entries name).
b2a_status create_cache(b2a_ctx* ctx, int num_layers, int num_kv_heads, int head_dim, int capacity, int batch,
                        b2a_dtype dtype, int page_size, int num_pages, b2a_kvcache** out) {
  if (out == nullptr) return fail(B2A_EINVAL, "null output pointer");
  *out = nullptr;
  // src/cpu/cache.js:24-26
  if (capacity < 1) return fail(B2A_ERANGE, "cache capacity must be a positive integer, got %d", capacity);
  if (num_layers < 1 || num_kv_heads < 1 || head_dim < 2 || head_dim % 8 != 0 || batch < 1) {
    return fail(B2A_EINVAL, "bad cache shape: layers %d, kv heads %d, head_dim %d, batch %d", num_layers,
                num_kv_heads, head_dim, batch);
  }
  if (!valid_dtype(dtype)) return fail(B2A_EINVAL, "unknown dtype %d", static_cast<int>(dtype));
  b2a_pagepool* pool = nullptr;
  if (page_size != 0) {
    b2a_status s = b2a_pagepool_create(num_pages, page_size, batch, capacity, &pool);
    if (s != B2A_OK) return s;
    // every pool row must be addressable by a 32-bit tensor-map coordinate
    const int64_t rows = (static_cast<int64_t>(num_pages) + 1) * num_layers * num_kv_heads * page_size;
    if (rows >= (1ll << 31)) {
      b2a_pagepool_destroy(pool);
      return fail(B2A_EINVAL, "paged cache of %d pages of %d positions is too large (%lld rows)", num_pages,
                  page_size, static_cast<long long>(rows));
    }
  }
  CallGuard g(ctx);
  if (!g.ok()) {
    b2a_pagepool_destroy(pool);
    return g.busy_status();
  }
  b2a_kvcache* c = new (std::nothrow) b2a_kvcache();
  c->ctx = ctx;
  c->device = ctx->device;
  c->layers = num_layers;
  c->kv_heads = num_kv_heads;
  c->head_dim = head_dim;
  c->capacity = capacity;
  c->batch = batch;
  c->dtype = dtype;
  const int block = page_size != 0 ? page_size : capacity;   // positions per block of the pools
  const int64_t units = page_size != 0 ? static_cast<int64_t>(num_pages) + 1 : batch;
  c->s_head = static_cast<int64_t>(block) * head_dim;
  c->s_layer = c->s_head * num_kv_heads;
  c->s_seq = c->s_layer * num_layers;
  c->len.assign(batch, 0);
  if (page_size != 0) {
    c->pool = pool;
    c->page_size = page_size;
    c->page_shift = 0;
    while ((1 << c->page_shift) < page_size) c->page_shift++;
    c->num_pages = num_pages;
    c->max_pages = static_cast<int>((static_cast<int64_t>(capacity) + page_size - 1) / page_size);
  }
  const size_t bytes = static_cast<size_t>(c->s_seq) * units * dtype_size(dtype);
  cudaError_t e = cudaMalloc(&c->d_k, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&c->d_v, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&c->d_len, sizeof(int32_t) * batch);
  if (e == cudaSuccess) e = cudaMemsetAsync(c->d_k, 0, bytes, ctx->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(c->d_v, 0, bytes, ctx->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(c->d_len, 0, sizeof(int32_t) * batch, ctx->stream);
  if (e == cudaSuccess && c->pool != nullptr) {
    const size_t tbytes = sizeof(int32_t) * static_cast<size_t>(batch) * c->max_pages;
    e = cudaMalloc(&c->d_pages, tbytes);
    // every entry starts at the scratch page (the host rows hold the same)
    if (e == cudaSuccess) e = cudaMemcpyAsync(c->d_pages, pool_row(c->pool, 0), tbytes, cudaMemcpyHostToDevice,
                                              ctx->stream);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    if (c->d_k) cudaFree(c->d_k);
    if (c->d_v) cudaFree(c->d_v);
    if (c->d_len) cudaFree(c->d_len);
    if (c->d_pages) cudaFree(c->d_pages);
    b2a_pagepool_destroy(c->pool);
    delete c;
    return cuda_fail(e, "allocating the KV cache");
  }
  if (dtype != B2A_F32 && head_dim == 64) {
    const uint64_t rows = static_cast<uint64_t>(units) * num_layers * num_kv_heads * block;
    c->has_tmaps = encode_pool_map(&c->tmap_k, c->d_k, rows, dtype) && encode_pool_map(&c->tmap_v, c->d_v, rows, dtype);
  }
  *out = c;
  return B2A_OK;
}

}  // namespace
}  // namespace b2a

extern "C" {

b2a_status b2a_kvcache_create(b2a_ctx* ctx, int num_layers, int num_kv_heads, int head_dim, int capacity, int batch,
                              b2a_dtype dtype, b2a_kvcache** out) {
  return create_cache(ctx, num_layers, num_kv_heads, head_dim, capacity, batch, dtype, 0, 0, out);
}

b2a_status b2a_kvcache_create_paged(b2a_ctx* ctx, int num_layers, int num_kv_heads, int head_dim, int capacity,
                                    int batch, b2a_dtype dtype, int page_size, int num_pages, b2a_kvcache** out) {
  if (out != nullptr) *out = nullptr;
  if (page_size == 0) return fail(B2A_EINVAL, "page size must be a power of two of at least 128 positions, got 0");
  return create_cache(ctx, num_layers, num_kv_heads, head_dim, capacity, batch, dtype, page_size, num_pages, out);
}

b2a_status b2a_kvcache_destroy(b2a_kvcache* c) {
  if (c == nullptr) return B2A_OK;
  cudaSetDevice(c->device);
  cudaFree(c->d_k);
  cudaFree(c->d_v);
  cudaFree(c->d_len);
  if (c->d_pages) cudaFree(c->d_pages);
  b2a_pagepool_destroy(c->pool);
  delete c;
  return B2A_OK;
}

b2a_status b2a_kvcache_allocate(b2a_kvcache* c, int seq_idx, int count, int* at) {
  if (c == nullptr || at == nullptr) return fail(B2A_EINVAL, "null argument");
  if (seq_idx < 0 || seq_idx >= c->batch) return fail(B2A_EINVAL, "sequence %d out of range [0, %d)", seq_idx, c->batch);
  if (count < 0) return fail(B2A_EINVAL, "count must be non-negative, got %d", count);
  const int len = c->len[seq_idx];
  // src/cpu/cache.js:53-58
  if (static_cast<int64_t>(len) + count > c->capacity) {
    return fail(B2A_ERANGE, "cache holds %d of %d positions; cannot add %d more", len, c->capacity, count);
  }
  if (c->pool != nullptr) {   // a paged cache backs the reserved positions now
    CallGuard g(c->ctx);
    if (!g.ok()) return g.busy_status();
    b2a_status s = cache_reserve1(c, seq_idx, len + count);
    if (s != B2A_OK) return s;
  }
  *at = len;
  return B2A_OK;
}

b2a_status b2a_kvcache_commit(b2a_kvcache* c, int seq_idx, int count) {
  if (c == nullptr) return fail(B2A_EINVAL, "null cache");
  if (seq_idx < -1 || seq_idx >= c->batch) return fail(B2A_EINVAL, "sequence %d out of range", seq_idx);
  for (int b = 0; b < c->batch; b++) {
    if (seq_idx >= 0 && b != seq_idx) continue;
    if (static_cast<int64_t>(c->len[b]) + count > c->capacity || c->len[b] + count < 0) {
      return fail(B2A_ERANGE, "cache holds %d of %d positions; cannot add %d more", c->len[b], c->capacity, count);
    }
  }
  CallGuard g(c->ctx);
  if (!g.ok()) return g.busy_status();
  if (c->pool != nullptr) {
    std::vector<int32_t> want(c->batch);
    for (int b = 0; b < c->batch; b++) want[b] = (seq_idx >= 0 && b != seq_idx) ? 0 : c->len[b] + count;
    b2a_status s = cache_reserve(c, 0, c->batch, want.data());
    if (s != B2A_OK) return s;
  }
  for (int b = 0; b < c->batch; b++) {
    if (seq_idx >= 0 && b != seq_idx) continue;
    c->len[b] += count;
  }
  cudaError_t e = launch_lengths_update(c->d_len, seq_idx, c->batch, count, 0, c->ctx->stream);
  if (e != cudaSuccess) return cuda_fail(e, "updating the device lengths");
  return B2A_OK;
}

b2a_status b2a_kvcache_length(const b2a_kvcache* c, int seq_idx, int* length) {
  if (c == nullptr || length == nullptr) return fail(B2A_EINVAL, "null argument");
  if (seq_idx < 0 || seq_idx >= c->batch) return fail(B2A_EINVAL, "sequence %d out of range [0, %d)", seq_idx, c->batch);
  *length = c->len[seq_idx];
  return B2A_OK;
}

b2a_status b2a_kvcache_set_lengths(b2a_kvcache* c, const int32_t* lengths) {
  if (c == nullptr || lengths == nullptr) return fail(B2A_EINVAL, "null argument");
  for (int b = 0; b < c->batch; b++) {
    if (lengths[b] < 0 || lengths[b] > c->capacity) {
      return fail(B2A_ERANGE, "length %d of sequence %d outside [0, %d]", lengths[b], b, c->capacity);
    }
  }
  CallGuard g(c->ctx);
  if (!g.ok()) return g.busy_status();
  b2a_status s = cache_reserve(c, 0, c->batch, lengths);
  if (s != B2A_OK) return s;
  for (int b = 0; b < c->batch; b++) c->len[b] = lengths[b];
  B2A_CUDA(cudaMemcpyAsync(c->d_len, c->len.data(), sizeof(int32_t) * c->batch, cudaMemcpyHostToDevice,
                           c->ctx->stream),
           "uploading lengths");
  B2A_CUDA(cudaStreamSynchronize(c->ctx->stream), "uploading lengths");
  return B2A_OK;
}

b2a_status b2a_kvcache_reset(b2a_kvcache* c, int seq_idx) {
  if (c == nullptr) return fail(B2A_EINVAL, "null cache");
  if (seq_idx < -1 || seq_idx >= c->batch) return fail(B2A_EINVAL, "sequence %d out of range", seq_idx);
  CallGuard g(c->ctx);
  if (!g.ok()) return g.busy_status();
  for (int b = 0; b < c->batch; b++) {
    if (seq_idx >= 0 && b != seq_idx) continue;
    c->len[b] = 0;
  }
  b2a_status s = cache_release(c, seq_idx);   // a paged cache gives the sequence's pages back
  if (s != B2A_OK) return s;
  cudaError_t e = launch_lengths_update(c->d_len, seq_idx, c->batch, 0, 1, c->ctx->stream);
  if (e != cudaSuccess) return cuda_fail(e, "resetting the device lengths");
  return B2A_OK;
}

b2a_status b2a_kvcache_byte_length(const b2a_kvcache* c, size_t* bytes) {
  if (c == nullptr || bytes == nullptr) return fail(B2A_EINVAL, "null argument");
  const size_t units = c->pool != nullptr ? static_cast<size_t>(c->num_pages) + 1 : static_cast<size_t>(c->batch);
  *bytes = static_cast<size_t>(c->s_seq) * units * dtype_size(c->dtype) * 2;
  return B2A_OK;
}

b2a_status b2a_kvcache_pools(const b2a_kvcache* c, void** keys, void** values, int64_t strides[4]) {
  if (c == nullptr) return fail(B2A_EINVAL, "null cache");
  if (keys) *keys = c->d_k;
  if (values) *values = c->d_v;
  if (strides) {
    strides[0] = c->s_seq;
    strides[1] = c->s_layer;
    strides[2] = c->s_head;
    strides[3] = c->head_dim;
  }
  return B2A_OK;
}

b2a_status b2a_kvcache_write_at(b2a_ctx* ctx, b2a_kvcache* c, int layer, int seq_idx, int at, const void* keys,
                                const void* values, b2a_dtype src_dtype, int count, int flags) {
  if (c == nullptr || keys == nullptr || values == nullptr) return fail(B2A_EINVAL, "null argument");
  if (!valid_dtype(src_dtype)) return fail(B2A_EINVAL, "unknown dtype %d", static_cast<int>(src_dtype));
  if (layer < 0 || layer >= c->layers) return fail(B2A_EINVAL, "layer %d out of range [0, %d)", layer, c->layers);
  if (seq_idx < 0 || seq_idx >= c->batch) return fail(B2A_EINVAL, "sequence %d out of range [0, %d)", seq_idx, c->batch);
  if (count < 0 || at < 0 || static_cast<int64_t>(at) + count > c->capacity) {
    return fail(B2A_ERANGE, "positions %d..%d outside the %d-position cache", at, at + count - 1, c->capacity);
  }
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  if (count > 0) {
    b2a_status s = cache_reserve1(c, seq_idx, at + count);
    if (s != B2A_OK) return s;
  }
  const size_t bytes = static_cast<size_t>(count) * c->kv_heads * c->head_dim * dtype_size(src_dtype);
  const void* dk = keys;
  const void* dv = values;
  if (flags == B2A_HOST) {
    Stage st;
    int ik = st.add(bytes), iv = st.add(bytes);
    b2a_status s = ensure_buffer(&ctx->d_stage, &ctx->d_stage_bytes, st.total, "allocating staging");
    if (s != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, ik), keys, bytes)) != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, iv), values, bytes)) != B2A_OK) return s;
    dk = st.ptr(ctx, ik);
    dv = st.ptr(ctx, iv);
  }
  cudaError_t e;
  {
    KernelTimer kt(ctx, K_WRITE_AT);
    e = launch_write_at(c, layer, seq_idx, at, dk, dv, static_cast<int>(src_dtype), count, ctx->stream);
  }
  if (e != cudaSuccess) return cuda_fail(e, "launching writeAt");
  if (flags == B2A_HOST) return d2h_sync(ctx, nullptr, nullptr, 0);
  return B2A_OK;
}

b2a_status b2a_kvcache_read(b2a_ctx* ctx, const b2a_kvcache* c, int layer, int seq_idx, int n, void* keys_out,
                            void* values_out, int flags) {
  if (c == nullptr || keys_out == nullptr || values_out == nullptr) return fail(B2A_EINVAL, "null argument");
  if (layer < 0 || layer >= c->layers) return fail(B2A_EINVAL, "layer %d out of range [0, %d)", layer, c->layers);
  if (seq_idx < 0 || seq_idx >= c->batch) return fail(B2A_EINVAL, "sequence %d out of range [0, %d)", seq_idx, c->batch);
  if (n < 0 || n > c->capacity) return fail(B2A_ERANGE, "cannot read %d positions of a %d-position cache", n, c->capacity);
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  const size_t es = dtype_size(c->dtype);
  const size_t head_bytes = static_cast<size_t>(n) * c->head_dim * es;
  const cudaMemcpyKind kind = flags == B2A_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
  if (c->pool != nullptr) {
    // one copy per (head, page); positions past the mapped pages read as zeros
    const int P = c->page_size;
    const int mapped = pool_mapped(c->pool, seq_idx);
    const int32_t* row = pool_row(c->pool, seq_idx);
    const size_t pos_bytes = static_cast<size_t>(c->head_dim) * es;
    const int backed = std::min(n, mapped * P);
    for (int h = 0; h < c->kv_heads; h++) {
      char* kd = static_cast<char*>(keys_out) + h * head_bytes;
      char* vd = static_cast<char*>(values_out) + h * head_bytes;
      for (int k = 0; k * P < backed; k++) {
        const int cnt = std::min(P, backed - k * P);
        const size_t off = (static_cast<size_t>(row[k]) * c->s_seq + static_cast<size_t>(layer) * c->s_layer +
                            static_cast<size_t>(h) * c->s_head) * es;
        B2A_CUDA(cudaMemcpyAsync(kd + k * P * pos_bytes, static_cast<const char*>(c->d_k) + off, cnt * pos_bytes, kind,
                                 ctx->stream), "reading keys");
        B2A_CUDA(cudaMemcpyAsync(vd + k * P * pos_bytes, static_cast<const char*>(c->d_v) + off, cnt * pos_bytes, kind,
                                 ctx->stream), "reading values");
      }
      if (backed < n) {
        const size_t zb = static_cast<size_t>(n - backed) * pos_bytes;
        if (flags == B2A_HOST) {
          std::memset(kd + backed * pos_bytes, 0, zb);
          std::memset(vd + backed * pos_bytes, 0, zb);
        } else {
          B2A_CUDA(cudaMemsetAsync(kd + backed * pos_bytes, 0, zb, ctx->stream), "reading keys");
          B2A_CUDA(cudaMemsetAsync(vd + backed * pos_bytes, 0, zb, ctx->stream), "reading values");
        }
      }
    }
    if (flags == B2A_HOST) B2A_CUDA(cudaStreamSynchronize(ctx->stream), "reading the cache");
    return B2A_OK;
  }
  for (int h = 0; h < c->kv_heads; h++) {
    const size_t off = (static_cast<size_t>(seq_idx) * c->s_seq + static_cast<size_t>(layer) * c->s_layer +
                        static_cast<size_t>(h) * c->s_head) * es;
    B2A_CUDA(cudaMemcpyAsync(static_cast<char*>(keys_out) + h * head_bytes, static_cast<const char*>(c->d_k) + off,
                             head_bytes, kind, ctx->stream), "reading keys");
    B2A_CUDA(cudaMemcpyAsync(static_cast<char*>(values_out) + h * head_bytes,
                             static_cast<const char*>(c->d_v) + off, head_bytes, kind, ctx->stream), "reading values");
  }
  if (flags == B2A_HOST) B2A_CUDA(cudaStreamSynchronize(ctx->stream), "reading the cache");
  return B2A_OK;
}

// ------------------------------------------------------------- append/rope --

b2a_status b2a_append_rope(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope, int layer, int seq_idx, const void* k,
                           const void* v, b2a_dtype src_dtype, int count, int flags) {
  if (c == nullptr || rope == nullptr || k == nullptr || v == nullptr) return fail(B2A_EINVAL, "null argument");
  if (!valid_dtype(src_dtype)) return fail(B2A_EINVAL, "unknown dtype %d", static_cast<int>(src_dtype));
  if (layer < 0 || layer >= c->layers) return fail(B2A_EINVAL, "layer %d out of range [0, %d)", layer, c->layers);
  if (seq_idx < 0 || seq_idx >= c->batch) return fail(B2A_EINVAL, "sequence %d out of range [0, %d)", seq_idx, c->batch);
  if (rope->head_dim != c->head_dim) return fail(B2A_EINVAL, "rope table head_dim differs from the cache's");
  if (count < 0) return fail(B2A_EINVAL, "count must be non-negative");
  const int past = c->len[seq_idx];
  if (static_cast<int64_t>(past) + count > c->capacity) {
    return fail(B2A_ERANGE, "cache holds %d of %d; cannot add %d", past, c->capacity, count);
  }
  if (static_cast<int64_t>(past) + count > rope->max_positions) {
    return fail(B2A_ERANGE, "position %d exceeds the %d-entry rope table", past + count, rope->max_positions);
  }
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  b2a_status rs = cache_reserve1(c, seq_idx, past + count);
  if (rs != B2A_OK) return rs;
  const size_t bytes = static_cast<size_t>(count) * c->kv_heads * c->head_dim * dtype_size(src_dtype);
  AttnParams p = base_params(ctx, c, rope);
  p.layer_begin = layer;
  p.in_dtype = static_cast<int>(src_dtype);
  p.k_new = k;
  p.v_new = v;
  if (flags == B2A_HOST) {
    Stage st;
    int ik = st.add(bytes), iv = st.add(bytes);
    b2a_status s = ensure_buffer(&ctx->d_stage, &ctx->d_stage_bytes, st.total, "allocating staging");
    if (s != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, ik), k, bytes)) != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, iv), v, bytes)) != B2A_OK) return s;
    p.k_new = st.ptr(ctx, ik);
    p.v_new = st.ptr(ctx, iv);
  }
  cudaError_t e;
  {
    KernelTimer kt(ctx, K_ROPE_APPEND);
    e = launch_rope_append(p, seq_idx, count, ctx->stream);
  }
  if (e != cudaSuccess) return cuda_fail(e, "launching the rope append");
  if (flags == B2A_HOST) return d2h_sync(ctx, nullptr, nullptr, 0);
  return B2A_OK;
}

// ------------------------------------------------------------------ decode --

b2a_status b2a_attention_decode(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope, int layer_begin, int num_layers,
                                int num_heads, const void* q, const void* k_new, const void* v_new,
                                b2a_dtype in_dtype, void* out, b2a_dtype out_dtype, int flags) {
  b2a_status s = check_cache_shape(c, rope, num_heads);
  if (s != B2A_OK) return s;
  if (q == nullptr || out == nullptr) return fail(B2A_EINVAL, "null q or out");
  if ((k_new == nullptr) != (v_new == nullptr)) return fail(B2A_EINVAL, "give both new keys and values, or neither");
  if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype)) return fail(B2A_EINVAL, "unknown dtype");
  if (layer_begin < 0 || num_layers < 1 || layer_begin + num_layers > c->layers) {
    return fail(B2A_EINVAL, "layers [%d, %d) outside the cache's %d", layer_begin, layer_begin + num_layers, c->layers);
  }
  int max_keys = 0;
  for (int b = 0; b < c->batch; b++) {
    const int past = c->len[b];
    // src/gpu/model.js:249-254
    if (past + 1 > c->capacity) {
      return fail(B2A_ERANGE, "cache holds %d of %d positions; cannot add 1 more", past, c->capacity);
    }
    if (past + 1 > rope->max_positions) {
      return fail(B2A_ERANGE, "position %d exceeds the %d-entry rope table", past + 1, rope->max_positions);
    }
    if (past + 1 > max_keys) max_keys = past + 1;
  }
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  if ((s = cache_reserve_all(c, 1)) != B2A_OK) return s;
  AttnParams p = base_params(ctx, c, rope);
  p.seq_begin = 0;
  p.batch = c->batch;
  p.num_layers = num_layers;
  p.layer_begin = layer_begin;
  p.tokens = 1;
  p.heads = num_heads;
  p.group = num_heads / c->kv_heads;
  p.in_dtype = static_cast<int>(in_dtype);
  p.q = q;
  p.k_new = k_new;
  p.v_new = v_new;
  p.horizon_extra = 1;
  const size_t ies = dtype_size(in_dtype);
  const size_t q_bytes = static_cast<size_t>(c->batch) * num_layers * num_heads * c->head_dim * ies;
  const size_t kv_bytes = static_cast<size_t>(c->batch) * num_layers * c->kv_heads * c->head_dim * ies;
  const size_t out_bytes = static_cast<size_t>(c->batch) * num_layers * num_heads * c->head_dim * dtype_size(out_dtype);
  void* dout = out;
  if (flags == B2A_HOST) {
    Stage st;
    int iq = st.add(q_bytes), ik = st.add(k_new ? kv_bytes : 0), iv = st.add(k_new ? kv_bytes : 0),
        io = st.add(out_bytes);
    if ((s = ensure_buffer(&ctx->d_stage, &ctx->d_stage_bytes, st.total, "allocating staging")) != B2A_OK) return s;
    p.q = st.ptr(ctx, iq);
    if (k_new) {
      p.k_new = st.ptr(ctx, ik);
      p.v_new = st.ptr(ctx, iv);
    }
    dout = st.ptr(ctx, io);
    return decode_host_pipelined(ctx, c, p, q, k_new, v_new, out, dout, static_cast<int>(out_dtype),
                                 static_cast<size_t>(num_layers) * num_heads * c->head_dim * ies,
                                 static_cast<size_t>(num_layers) * c->kv_heads * c->head_dim * ies,
                                 static_cast<size_t>(num_layers) * num_heads * c->head_dim * dtype_size(out_dtype), -1);
  }
  return run_split_kv(ctx, c, p, max_keys, dout, static_cast<int>(out_dtype), 0);
}

b2a_status b2a_attention_decode_host_async(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope, int layer_begin,
                                           int num_layers, int num_heads, const void* q, const void* k_new,
                                           const void* v_new, b2a_dtype in_dtype, void* out, b2a_dtype out_dtype) {
  b2a_status s = check_cache_shape(c, rope, num_heads);
  if (s != B2A_OK) return s;
  if (q == nullptr || out == nullptr) return fail(B2A_EINVAL, "null q or out");
  if ((k_new == nullptr) != (v_new == nullptr)) return fail(B2A_EINVAL, "give both new keys and values, or neither");
  if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype)) return fail(B2A_EINVAL, "unknown dtype");
  if (layer_begin < 0 || num_layers < 1 || layer_begin + num_layers > c->layers) {
    return fail(B2A_EINVAL, "layers [%d, %d) outside the cache's %d", layer_begin, layer_begin + num_layers, c->layers);
  }
  for (int b = 0; b < c->batch; b++) {
    const int past = c->len[b];
    if (past + 1 > c->capacity) {
      return fail(B2A_ERANGE, "cache holds %d of %d positions; cannot add 1 more", past, c->capacity);
    }
    if (past + 1 > rope->max_positions) {
      return fail(B2A_ERANGE, "position %d exceeds the %d-entry rope table", past + 1, rope->max_positions);
    }
  }
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  if ((s = cache_reserve_all(c, 1)) != B2A_OK) return s;
  const int slot = ctx->async_next;
  if (ctx->async_free[slot] == nullptr) {
    B2A_CUDA(cudaEventCreateWithFlags(&ctx->async_free[slot], cudaEventDisableTiming), "creating a slot event");
  }
  const size_t ies = dtype_size(in_dtype);
  const size_t q_bytes = static_cast<size_t>(c->batch) * num_layers * num_heads * c->head_dim * ies;
  const size_t kv_bytes = static_cast<size_t>(c->batch) * num_layers * c->kv_heads * c->head_dim * ies;
  const size_t out_bytes = static_cast<size_t>(c->batch) * num_layers * num_heads * c->head_dim * dtype_size(out_dtype);
  Stage st;
  int iq = st.add(q_bytes), ik = st.add(k_new ? kv_bytes : 0), iv = st.add(k_new ? kv_bytes : 0),
      io = st.add(out_bytes);
  // growing a slot frees it first, which waits for every call still using it
  if ((s = ensure_buffer(&ctx->d_async[slot], &ctx->d_async_bytes[slot], st.total, "allocating async staging")) !=
      B2A_OK) {
    return s;
  }
  char* base = static_cast<char*>(ctx->d_async[slot]);
  AttnParams p = base_params(ctx, c, rope);
  p.seq_begin = 0;
  p.batch = c->batch;
  p.num_layers = num_layers;
  p.layer_begin = layer_begin;
  p.tokens = 1;
  p.heads = num_heads;
  p.group = num_heads / c->kv_heads;
  p.in_dtype = static_cast<int>(in_dtype);
  p.q = base + st.offsets[iq];
  p.k_new = k_new ? base + st.offsets[ik] : nullptr;
  p.v_new = k_new ? base + st.offsets[iv] : nullptr;
  p.horizon_extra = 1;
  s = decode_host_pipelined(ctx, c, p, q, k_new, v_new, out, base + st.offsets[io], static_cast<int>(out_dtype),
                            static_cast<size_t>(num_layers) * num_heads * c->head_dim * ies,
                            static_cast<size_t>(num_layers) * c->kv_heads * c->head_dim * ies,
                            static_cast<size_t>(num_layers) * num_heads * c->head_dim * dtype_size(out_dtype), slot);
  if (s == B2A_OK) ctx->async_next = slot ^ 1;
  return s;
}

}  // extern "C"

namespace b2a {

b2a_status attn_decode_device(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope, int layer, int num_heads,
                              const void* q, const void* k_new, const void* v_new, b2a_dtype in_dtype, void* out,
                              b2a_dtype out_dtype) {
  int max_keys = 0;
  for (int b = 0; b < c->batch; b++) max_keys = std::max(max_keys, c->len[b] + 1);
  b2a_status s = cache_reserve_all(c, 1);
  if (s != B2A_OK) return s;
  AttnParams p = base_params(ctx, c, rope);
  p.seq_begin = 0;
  p.batch = c->batch;
  p.num_layers = 1;
  p.layer_begin = layer;
  p.tokens = 1;
  p.heads = num_heads;
  p.group = num_heads / c->kv_heads;
  p.in_dtype = static_cast<int>(in_dtype);
  p.q = q;
  p.k_new = k_new;
  p.v_new = v_new;
  p.horizon_extra = 1;
  return run_split_kv(ctx, c, p, max_keys, out, static_cast<int>(out_dtype), 0);
}

}  // namespace b2a

extern "C" {

// ----------------------------------------------------------------- prefill --

namespace {
// Query tiles per CTA of the f16-cache prefill: the two-tile kernel halves the
// CTA count, which pays once there are at least two CTAs per SM to spread
// (measured: one-tile faster at S <= 2048, two-tile faster at S >= 8192 for 14
// heads). B2A_PREFILL_TILES=1 or 2 forces a kernel (read on every call, so a
// process can compare both).
int prefill_tiles_per_cta(const b2a_ctx* ctx, int count, int heads) {
  const char* v = std::getenv("B2A_PREFILL_TILES");
  if (v != nullptr && (v[0] == '1' || v[0] == '2') && v[1] == 0) return v[0] - '0';
  const int64_t ctas = static_cast<int64_t>((count + 127) / 128) * heads;
  return ctas >= 2LL * ctx->sm_count ? 2 : 1;
}
}  // namespace

b2a_status b2a_attention_prefill(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope, int layer, int seq_idx,
                                 int num_heads, const void* q, const void* k, const void* v, b2a_dtype in_dtype,
                                 int count, void* out, b2a_dtype out_dtype, int flags) {
  b2a_status s = check_cache_shape(c, rope, num_heads);
  if (s != B2A_OK) return s;
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr) return fail(B2A_EINVAL, "null argument");
  if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype)) return fail(B2A_EINVAL, "unknown dtype");
  if (layer < 0 || layer >= c->layers) return fail(B2A_EINVAL, "layer %d out of range [0, %d)", layer, c->layers);
  if (seq_idx < 0 || seq_idx >= c->batch) return fail(B2A_EINVAL, "sequence %d out of range [0, %d)", seq_idx, c->batch);
  if (count < 1) return fail(B2A_EINVAL, "forward: need at least one token");
  const int past = c->len[seq_idx];
  if (static_cast<int64_t>(past) + count > c->capacity) {
    return fail(B2A_ERANGE, "cache holds %d of %d positions; cannot add %d more", past, c->capacity, count);
  }
  if (static_cast<int64_t>(past) + count > rope->max_positions) {
    return fail(B2A_ERANGE, "position %d exceeds the %d-entry rope table", past + count, rope->max_positions);
  }
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  const size_t ies = dtype_size(in_dtype);
  const size_t q_bytes = static_cast<size_t>(count) * num_heads * c->head_dim * ies;
  const size_t kv_bytes = static_cast<size_t>(count) * c->kv_heads * c->head_dim * ies;
  const size_t out_bytes = static_cast<size_t>(count) * num_heads * c->head_dim * dtype_size(out_dtype);
  void* dout = out;
  if (flags == B2A_HOST) {
    Stage st;
    int iq = st.add(q_bytes), ik = st.add(kv_bytes), iv = st.add(kv_bytes), io = st.add(out_bytes);
    if ((s = ensure_buffer(&ctx->d_stage, &ctx->d_stage_bytes, st.total, "allocating staging")) != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, iq), q, q_bytes)) != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, ik), k, kv_bytes)) != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, iv), v, kv_bytes)) != B2A_OK) return s;
    q = st.ptr(ctx, iq);
    k = st.ptr(ctx, ik);
    v = st.ptr(ctx, iv);
    dout = st.ptr(ctx, io);
  }
  if ((s = attn_prefill_device(ctx, c, rope, layer, seq_idx, num_heads, q, k, v, in_dtype, count, dout, out_dtype)) !=
      B2A_OK) {
    return s;
  }
  if (flags == B2A_HOST) return d2h_sync(ctx, out, dout, out_bytes);
  return B2A_OK;
}

}  // extern "C"

namespace b2a {

b2a_status attn_prefill_device(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope, int layer, int seq_idx,
                               int num_heads, const void* q, const void* k, const void* v, b2a_dtype in_dtype,
                               int count, void* dout, b2a_dtype out_dtype, int nseq) {
  b2a_status s;
  int past = 0;   // the longest past among the call's sequences
  for (int b = 0; b < nseq; b++) past = std::max(past, c->len[seq_idx + b]);
  if (c->pool != nullptr) {
    std::vector<int32_t> want(nseq);
    for (int b = 0; b < nseq; b++) want[b] = c->len[seq_idx + b] + count;
    if ((s = cache_reserve(c, seq_idx, nseq, want.data())) != B2A_OK) return s;
  }
  AttnParams p = base_params(ctx, c, rope);
  p.seq_begin = seq_idx;
  p.batch = nseq;
  p.num_layers = 1;
  p.layer_begin = layer;
  p.tokens = count;
  p.heads = num_heads;
  p.group = num_heads / c->kv_heads;
  p.in_dtype = static_cast<int>(in_dtype);
  p.q = q;
  p.k_new = k;
  p.v_new = v;
  p.horizon_extra = 1;
  if (c->has_tmaps) {
    p.tmap_k = &c->tmap_k;
    p.tmap_v = &c->tmap_v;
  }
  // The tensor-core kernels (f16 cache) take their query tiles by TMA from
  // RoPE(q) rows that the append kernel writes (the one-tile kernel with a
  // bf16 cache stages its own: it splits each query into two bf16 parts).
  CUtensorMap qmap;
  AttnParams attn = p;   // as the attention kernels see it: the new rows are in the cache
  attn.k_new = nullptr;
  attn.v_new = nullptr;
  const bool rows_ok = c->dtype == B2A_F16 && c->head_dim == 64 && c->has_tmaps;
  attn.tmap_q = rows_ok ? &qmap : nullptr;   // the map is encoded below, only if it is used
  bool pair = prefill_pair_supported(attn) && prefill_tiles_per_cta(ctx, count, num_heads * nseq) == 2;
  if (pair || (rows_ok && prefill_tc_supported(attn))) {
    const size_t rows = static_cast<size_t>(nseq) * count;
    if ((s = ensure_buffer(&ctx->d_qrot, &ctx->d_qrot_bytes, rows * num_heads * 64 * sizeof(uint16_t),
                           "allocating rotated queries")) != B2A_OK) {
      return s;
    }
    if (encode_query_map(&qmap, ctx->d_qrot, rows, num_heads)) {
      p.q_rot = static_cast<uint16_t*>(ctx->d_qrot);
      p.tmap_q = &qmap;
    } else {
      pair = false;   // the one-tile kernel stages its own query tiles
    }
  }
  // RoPE(K) + append first (src/cpu/model.js:116 writes before attending), then
  // causal attention over past+count, with RoPE(Q) done by the append kernel
  // (tensor-core kernels, f16 cache) or fused into the Q load (the others).
  cudaError_t e;
  {
    KernelTimer kt(ctx, K_ROPE_APPEND);
    e = launch_rope_append(p, seq_idx, count, ctx->stream, nseq);
  }
  if (e != cudaSuccess) return cuda_fail(e, "launching the rope append");
  p.k_new = nullptr;
  p.v_new = nullptr;
  if (pair) {
    // tensor-core causal attention, two heads' 128-query tiles per CTA (f16 cache)
    CUtensorMap omap;
    if (encode_output_map(&omap, dout, nseq, count, num_heads, static_cast<int>(out_dtype))) p.tmap_o = &omap;
    {
      KernelTimer kt(ctx, K_PREFILL_PAIR);
      e = launch_prefill_pair(p, dout, static_cast<int>(out_dtype), ctx->stream);
    }
    if (e != cudaSuccess) return cuda_fail(e, "launching the tensor-core prefill");
  } else if (prefill_tc_supported(p)) {
    // tensor-core causal attention: one CTA per (128-query tile, head), no split
    {
      KernelTimer kt(ctx, K_PREFILL_TC);
      e = launch_prefill_tc(p, dout, static_cast<int>(out_dtype), ctx->stream);
    }
    if (e != cudaSuccess) return cuda_fail(e, "launching the tensor-core prefill");
  } else if ((s = run_split_kv(ctx, c, p, past + count, dout, static_cast<int>(out_dtype), 0)) != B2A_OK) {
    return s;
  }
  return B2A_OK;
}

}  // namespace b2a

extern "C" {

b2a_status b2a_attention_prefill_batch(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope, int layer, int seq_begin,
                                       int nseq, int num_heads, const void* q, const void* k, const void* v,
                                       b2a_dtype in_dtype, int count, void* out, b2a_dtype out_dtype, int flags) {
  b2a_status s = check_cache_shape(c, rope, num_heads);
  if (s != B2A_OK) return s;
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr) return fail(B2A_EINVAL, "null argument");
  if (!valid_dtype(in_dtype) || !valid_dtype(out_dtype)) return fail(B2A_EINVAL, "unknown dtype");
  if (layer < 0 || layer >= c->layers) return fail(B2A_EINVAL, "layer %d out of range [0, %d)", layer, c->layers);
  if (nseq < 1 || seq_begin < 0 || seq_begin + nseq > c->batch) {
    return fail(B2A_EINVAL, "sequences [%d, %d) out of range [0, %d)", seq_begin, seq_begin + nseq, c->batch);
  }
  if (count < 1) return fail(B2A_EINVAL, "forward: need at least one token");
  for (int b = seq_begin; b < seq_begin + nseq; b++) {
    const int past = c->len[b];
    // src/gpu/model.js:249-254, per sequence
    if (static_cast<int64_t>(past) + count > c->capacity) {
      return fail(B2A_ERANGE, "cache holds %d of %d positions; cannot add %d more", past, c->capacity, count);
    }
    if (static_cast<int64_t>(past) + count > rope->max_positions) {
      return fail(B2A_ERANGE, "position %d exceeds the %d-entry rope table", past + count, rope->max_positions);
    }
  }
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  const size_t ies = dtype_size(in_dtype);
  const size_t q_bytes = static_cast<size_t>(nseq) * count * num_heads * c->head_dim * ies;
  const size_t kv_bytes = static_cast<size_t>(nseq) * count * c->kv_heads * c->head_dim * ies;
  const size_t out_bytes = static_cast<size_t>(nseq) * count * num_heads * c->head_dim * dtype_size(out_dtype);
  void* dout = out;
  if (flags == B2A_HOST) {
    Stage st;
    int iq = st.add(q_bytes), ik = st.add(kv_bytes), iv = st.add(kv_bytes), io = st.add(out_bytes);
    if ((s = ensure_buffer(&ctx->d_stage, &ctx->d_stage_bytes, st.total, "allocating staging")) != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, iq), q, q_bytes)) != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, ik), k, kv_bytes)) != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, iv), v, kv_bytes)) != B2A_OK) return s;
    q = st.ptr(ctx, iq);
    k = st.ptr(ctx, ik);
    v = st.ptr(ctx, iv);
    dout = st.ptr(ctx, io);
  }
  if ((s = attn_prefill_device(ctx, c, rope, layer, seq_begin, num_heads, q, k, v, in_dtype, count, dout, out_dtype,
                               nseq)) != B2A_OK) {
    return s;
  }
  if (flags == B2A_HOST) return d2h_sync(ctx, out, dout, out_bytes);
  return B2A_OK;
}

// ----------------------------------------------------- groupedAttention drop-in --

b2a_status b2a_grouped_attention(b2a_ctx* ctx, const float* q, const float* keys, const float* values, float* out,
                                 float* scores, int seq, int past, int num_heads, int num_kv_heads, int head_dim,
                                 int flags) {
  (void)scores;
  if (q == nullptr || keys == nullptr || values == nullptr || out == nullptr) return fail(B2A_EINVAL, "null argument");
  if (seq < 0 || past < 0 || num_heads < 1 || num_kv_heads < 1 || num_heads % num_kv_heads != 0) {
    return fail(B2A_EINVAL, "bad attention shape: seq %d, past %d, heads %d/%d", seq, past, num_heads, num_kv_heads);
  }
  if (head_dim < 1 || head_dim > 256) return fail(B2A_EINVAL, "head_dim must be in [1, 256], got %d", head_dim);
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  if (seq == 0) return B2A_OK;
  const size_t q_bytes = static_cast<size_t>(seq) * num_heads * head_dim * 4;
  const size_t kv_bytes = static_cast<size_t>(past + seq) * num_kv_heads * head_dim * 4;
  const float* dq = q;
  const float* dk = keys;
  const float* dv = values;
  float* dout = out;
  if (flags == B2A_HOST) {
    Stage st;
    int iq = st.add(q_bytes), ik = st.add(kv_bytes), iv = st.add(kv_bytes), io = st.add(q_bytes);
    b2a_status s = ensure_buffer(&ctx->d_stage, &ctx->d_stage_bytes, st.total, "allocating staging");
    if (s != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, iq), q, q_bytes)) != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, ik), keys, kv_bytes)) != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, iv), values, kv_bytes)) != B2A_OK) return s;
    dq = static_cast<const float*>(st.ptr(ctx, iq));
    dk = static_cast<const float*>(st.ptr(ctx, ik));
    dv = static_cast<const float*>(st.ptr(ctx, iv));
    dout = static_cast<float*>(st.ptr(ctx, io));
  }
  cudaError_t e;
  {
    KernelTimer kt(ctx, K_GROUPED);
    e = launch_grouped_generic(dq, dk, dv, dout, seq, past, num_heads, num_kv_heads, head_dim, ctx->stream);
  }
  if (e != cudaSuccess) return cuda_fail(e, "launching groupedAttention");
  if (flags == B2A_HOST) return d2h_sync(ctx, out, dout, q_bytes);
  return B2A_OK;
}

// --------------------------------------------------------- split-KV partials --

b2a_status b2a_attention_decode_partial(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope, int layer, int num_heads,
                                        const void* q, const void* k_new, const void* v_new, b2a_dtype in_dtype,
                                        const int32_t* q_positions, float* partial, int flags) {
  if (partial == nullptr) return fail(B2A_EINVAL, "null argument");
  return decode_positions(ctx, c, rope, layer, 1, num_heads, q, k_new, v_new, in_dtype, q_positions, nullptr, partial,
                          B2A_F32, flags);
}

b2a_status b2a_attention_decode_partial_layers(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope, int layer_begin,
                                               int num_layers, int num_heads, const void* q, const void* k_new,
                                               const void* v_new, b2a_dtype in_dtype, const int32_t* q_positions,
                                               float* partial, int flags) {
  if (partial == nullptr) return fail(B2A_EINVAL, "null argument");
  return decode_positions(ctx, c, rope, layer_begin, num_layers, num_heads, q, k_new, v_new, in_dtype, q_positions,
                          nullptr, partial, B2A_F32, flags);
}

b2a_status b2a_quantize_int8_per_channel(const float* w, int rows, int cols, int8_t* codes, float* scales) {
  if (w == nullptr || codes == nullptr || scales == nullptr) return fail(B2A_EINVAL, "null argument");
  if (rows < 0 || cols < 0) return fail(B2A_EINVAL, "bad shape %d x %d", rows, cols);
  // src/core/quantize.js:36-58: the row peak over 127 in f64, stored f32; the
  // codes divide by the f64 scale and round half away from zero (C's round)
  for (int r = 0; r < rows; r++) {
    const float* row = w + static_cast<size_t>(r) * cols;
    double peak = 0.0;
    for (int c = 0; c < cols; c++) peak = std::max(peak, std::fabs(static_cast<double>(row[c])));
    const double scale = peak / 127.0;
    scales[r] = static_cast<float>(scale);
    int8_t* out = codes + static_cast<size_t>(r) * cols;
    if (scale == 0.0) {
      std::memset(out, 0, static_cast<size_t>(cols));
      continue;
    }
    const double inverse = 1.0 / scale;
    for (int c = 0; c < cols; c++) {
      const double level = std::round(static_cast<double>(row[c]) * inverse);
      out[c] = static_cast<int8_t>(std::min(127.0, std::max(-127.0, level)));
    }
  }
  return B2A_OK;
}

b2a_status b2a_linear_int8(b2a_ctx* ctx, const int8_t* codes, const void* scales, b2a_dtype scale_dtype,
                           const void* bias, b2a_dtype bias_dtype, const void* x, b2a_dtype x_dtype, int rows,
                           int cols, int tokens, const void* residual, void* out, b2a_dtype out_dtype, int flags) {
  void* outs[1] = {out};
  const int seg_end[1] = {rows};
  return linear_int8(ctx, codes, scales, scale_dtype, bias, bias_dtype, x, x_dtype, rows, cols, tokens, residual,
                     outs, seg_end, 1, out_dtype, flags);
}

b2a_status b2a_qkv_int8(b2a_ctx* ctx, const int8_t* codes, const void* scales, b2a_dtype scale_dtype,
                        const void* bias, b2a_dtype bias_dtype, const void* x, b2a_dtype x_dtype, int hidden,
                        int q_rows, int kv_rows, int tokens, void* q_out, void* k_out, void* v_out,
                        b2a_dtype out_dtype, int flags) {
  if (q_rows < 1 || kv_rows < 1) return fail(B2A_EINVAL, "q rows %d and kv rows %d must be positive", q_rows, kv_rows);
  void* outs[3] = {q_out, k_out, v_out};
  const int seg_end[3] = {q_rows, q_rows + kv_rows, q_rows + 2 * kv_rows};
  return linear_int8(ctx, codes, scales, scale_dtype, bias, bias_dtype, x, x_dtype, q_rows + 2 * kv_rows, hidden,
                     tokens, nullptr, outs, seg_end, 3, out_dtype, flags);
}

b2a_status b2a_exchange_create(b2a_ctx* ctx, int world, int rank, int batch, int num_heads, int num_kv_heads,
                               b2a_exchange** out) {
  return b2a_exchange_create_layers(ctx, world, rank, batch, 1, num_heads, num_kv_heads, out);
}

b2a_status b2a_exchange_create_layers(b2a_ctx* ctx, int world, int rank, int batch, int num_layers, int num_heads,
                                      int num_kv_heads, b2a_exchange** out) {
  if (ctx == nullptr || out == nullptr) return fail(B2A_EINVAL, "null argument");
  *out = nullptr;
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world) {
    return fail(B2A_EINVAL, "rank %d of world %d: the exchange takes 1..%d ranks", rank, world, kMaxWorld);
  }
  if (batch < 1 || num_layers < 1 || num_kv_heads < 1 || num_heads < 1 || num_heads % num_kv_heads != 0) {
    return fail(B2A_EINVAL, "bad exchange shape: batch %d, layers %d, heads %d, kv heads %d", batch, num_layers,
                num_heads, num_kv_heads);
  }
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  b2a_exchange* ex = new (std::nothrow) b2a_exchange();
  if (ex == nullptr) return fail(B2A_ECUDA, "out of host memory for the exchange");
  ex->device = ctx->device;
  ex->world = world;
  ex->rank = rank;
  ex->batch = batch;
  ex->layers = num_layers;
  ex->heads = num_heads;
  ex->kv_heads = num_kv_heads;
  ex->rows = batch * num_layers * num_heads;
  ex->groups = batch * num_layers * num_kv_heads;
  const size_t x_bytes = 2ull * world * ex->rows * (64 + 4) * sizeof(uint64_t);
  ex->c_off = (x_bytes + 255) & ~size_t(255);
  ex->bytes = ex->c_off + 256;
  cudaError_t e = cudaMalloc(&ex->base, ex->bytes);
  if (e == cudaSuccess) e = cudaMemset(ex->base, 0, ex->bytes);
  if (e != cudaSuccess) {
    if (ex->base) cudaFree(ex->base);
    delete ex;
    return cuda_fail(e, "allocating the exchange buffer");
  }
  for (int r = 0; r < kMaxWorld; r++) ex->peer[r] = nullptr;
  ex->peer[rank] = ex->base;
  *out = ex;
  return B2A_OK;
}

b2a_status b2a_exchange_handle(const b2a_exchange* ex, void* handle) {
  if (ex == nullptr || handle == nullptr) return fail(B2A_EINVAL, "null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == B2A_EXCHANGE_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  cudaSetDevice(ex->device);
  B2A_CUDA(cudaIpcGetMemHandle(&h, ex->base), "exporting the exchange buffer");
  std::memcpy(handle, &h, sizeof(h));
  return B2A_OK;
}

b2a_status b2a_exchange_open(b2a_exchange* ex, const void* handles) {
  if (ex == nullptr || handles == nullptr) return fail(B2A_EINVAL, "null argument");
  cudaSetDevice(ex->device);
  for (int r = 0; r < ex->world; r++) {
    if (r == ex->rank || ex->peer[r] != nullptr) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const char*>(handles) + static_cast<size_t>(r) * sizeof(h), sizeof(h));
    void* ptr = nullptr;
    B2A_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess), "opening a peer's exchange buffer");
    ex->peer[r] = ptr;
    ex->opened[r] = true;
  }
  return B2A_OK;
}

b2a_status b2a_exchange_connect_local(b2a_exchange* ex, int peer, const b2a_exchange* other) {
  if (ex == nullptr || other == nullptr) return fail(B2A_EINVAL, "null argument");
  if (peer < 0 || peer >= ex->world || peer == ex->rank) return fail(B2A_EINVAL, "bad peer rank %d", peer);
  if (other->device != ex->device || other->bytes != ex->bytes || other->world != ex->world || other->rank != peer) {
    return fail(B2A_EINVAL, "exchange %d is not rank %d of the same shape on this device", other->rank, peer);
  }
  ex->peer[peer] = other->base;
  ex->opened[peer] = false;
  return B2A_OK;
}

b2a_status b2a_exchange_destroy(b2a_exchange* ex) {
  if (ex == nullptr) return B2A_OK;
  cudaSetDevice(ex->device);
  for (int r = 0; r < kMaxWorld; r++) {
    if (ex->opened[r] && ex->peer[r] != nullptr) cudaIpcCloseMemHandle(ex->peer[r]);
  }
  cudaFree(ex->base);
  delete ex;
  return B2A_OK;
}

b2a_status b2a_attention_decode_split(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope, int layer, int num_heads,
                                      const void* q, const void* k_new, const void* v_new, b2a_dtype in_dtype,
                                      const int32_t* q_positions, b2a_exchange* ex, void* out, b2a_dtype out_dtype,
                                      int flags) {
  return b2a_attention_decode_split_layers(ctx, c, rope, layer, 1, num_heads, q, k_new, v_new, in_dtype, q_positions,
                                           ex, out, out_dtype, flags);
}

b2a_status b2a_attention_decode_split_layers(b2a_ctx* ctx, b2a_kvcache* c, const b2a_rope* rope, int layer_begin,
                                             int num_layers, int num_heads, const void* q, const void* k_new,
                                             const void* v_new, b2a_dtype in_dtype, const int32_t* q_positions,
                                             b2a_exchange* ex, void* out, b2a_dtype out_dtype, int flags) {
  if (ex == nullptr || out == nullptr) return fail(B2A_EINVAL, "null argument");
  if (num_layers != ex->layers) {
    return fail(B2A_EINVAL, "the exchange was made for %d layers per call; the call has %d", ex->layers, num_layers);
  }
  if (!valid_dtype(out_dtype)) return fail(B2A_EINVAL, "unknown dtype");
  if (c != nullptr && (c->batch != ex->batch || c->kv_heads != ex->kv_heads || num_heads != ex->heads)) {
    return fail(B2A_EINVAL, "the exchange was made for batch %d, %d/%d heads; the call has batch %d, %d/%d", ex->batch,
                ex->heads, ex->kv_heads, c->batch, num_heads, c->kv_heads);
  }
  if (c != nullptr && c->device != ex->device) return fail(B2A_EINVAL, "the exchange lives on another device");
  for (int r = 0; r < ex->world; r++) {
    if (ex->peer[r] == nullptr) return fail(B2A_EINVAL, "exchange rank %d is not connected; open the handles first", r);
  }
  return decode_positions(ctx, c, rope, layer_begin, num_layers, num_heads, q, k_new, v_new, in_dtype, q_positions, ex,
                          out, out_dtype, flags);
}

b2a_status b2a_lse_combine(b2a_ctx* ctx, const float* partials, int num_parts, int batch, int num_heads, int head_dim,
                           void* out, b2a_dtype out_dtype, int flags) {
  if (partials == nullptr || out == nullptr) return fail(B2A_EINVAL, "null argument");
  if (num_parts < 1 || batch < 0 || num_heads < 1 || head_dim < 1 || head_dim > 128) {
    return fail(B2A_EINVAL, "bad combine shape: parts %d, batch %d, heads %d, head_dim %d", num_parts, batch,
                num_heads, head_dim);
  }
  if (!valid_dtype(out_dtype)) return fail(B2A_EINVAL, "unknown dtype");
  CallGuard g(ctx);
  if (!g.ok()) return g.busy_status();
  const int64_t rows = static_cast<int64_t>(batch) * num_heads;
  const size_t in_bytes = static_cast<size_t>(num_parts) * rows * (head_dim + 4) * 4;
  const size_t out_bytes = static_cast<size_t>(rows) * head_dim * dtype_size(out_dtype);
  const float* dpart = partials;
  void* dout = out;
  if (flags == B2A_HOST) {
    Stage st;
    int ip = st.add(in_bytes), io = st.add(out_bytes);
    b2a_status s = ensure_buffer(&ctx->d_stage, &ctx->d_stage_bytes, st.total, "allocating staging");
    if (s != B2A_OK) return s;
    if ((s = h2d(ctx, st.ptr(ctx, ip), partials, in_bytes)) != B2A_OK) return s;
    dpart = static_cast<const float*>(st.ptr(ctx, ip));
    dout = st.ptr(ctx, io);
  }
  CombineParams cp{};
  cp.partial = dpart;
  cp.rows = rows;
  cp.nchunks = num_parts;
  cp.head_dim = head_dim;
  cp.part_stride_rows = static_cast<int>(rows);
  cp.out = dout;
  cp.out_dtype = static_cast<int>(out_dtype);
  cp.mode = 0;
  cudaError_t e = launch_combine(cp, ctx->stream);
  if (e != cudaSuccess) return cuda_fail(e, "launching the combine");
  if (flags == B2A_HOST) return d2h_sync(ctx, out, dout, out_bytes);
  return B2A_OK;
}

}  // extern "C"
