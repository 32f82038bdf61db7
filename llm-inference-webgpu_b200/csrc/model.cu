// The Qwen2 decoder around the attention path (include/b2a.h, b2a_model_*):
// ReferenceModel.forward / generate (src/cpu/model.js:55-187) and
// GpuModel.forward (src/gpu/model.js:227-400), with int8 weights holding one
// scale per output row.
//
// Device layout: all weights in one allocation, per layer
//   qkv codes [hidden + 2 kv_dim][hidden] (q rows, k rows, v rows; one
//   projection with three outputs), o codes [hidden][hidden], gate and up
//   codes interleaved by row [2 intermediate][hidden] (gate row i at 2i, up
//   row i at 2i+1: one projection whose consecutive outputs pair up for SwiGLU),
//   down codes [hidden][intermediate], then their scales, the qkv bias and the
//   two norm gains;
// then the tied embedding [vocab][hidden] with its scales and the final norm.
// Activations (x, the normed rows, q/k/v in f16, attention output, gate, up)
// grow with the longest forward; the KV cache holds one sequence in f16.
//
// One forward (the reference's order, every launch on the context's stream,
// each a programmatic dependent of the one before):
//   embed -> per layer [rmsnorm, qkv projection (+bias) -> f16 q/k/v,
//   attention (decode kernel for one token, tensor-core prefill for several;
//   RoPE and the KV append fused), o projection (+residual, in place),
//   rmsnorm, gate/up projection, swiglu, down projection (+residual)]
//   -> commit -> final rmsnorm of the last row -> tied output projection ->
//   argmax.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "b2a_internal.cuh"
#include "k_util.cuh"

struct b2a_model {
  b2a_ctx* ctx = nullptr;
  int device = 0;
  b2a_model_config cfg{};
  int capacity = 0;
  int kv_dim = 0, qkv_rows = 0;
  size_t ssz = 2;                        // bytes per scale
  b2a_kvcache* cache = nullptr;
  b2a_rope* rope = nullptr;
  void* d_weights = nullptr;
  struct Layer {
    int8_t *qkv, *o, *gu, *down;
    void *s_qkv, *s_o, *s_gu, *s_down;
    float *b_qkv, *n_in, *n_post;
    bool loaded;
  };
  std::vector<Layer> layers;
  int8_t* emb = nullptr;
  void* s_emb = nullptr;
  float* n_final = nullptr;
  bool emb_loaded = false, final_loaded = false;
  // activations for up to t_cap tokens per forward
  void* d_act = nullptr;
  int t_cap = 0;
  // gate: the interleaved gate/up outputs [T][2 inter]; up: silu(gate) * up [T][inter]
  float *x = nullptr, *nx = nullptr, *att = nullptr, *gate = nullptr, *up = nullptr;
  uint16_t *q = nullptr, *k = nullptr, *v = nullptr;
  // fixed buffers: logits, prompt tokens, generated tokens and their logits, argmax scratch
  void* d_fixed = nullptr;
  float* logits = nullptr;
  int32_t* tokens = nullptr;             // [capacity]
  int32_t* gen = nullptr;                // [capacity]
  float* best = nullptr;                 // [capacity]
  void* arg_scratch = nullptr;
  // the one-kernel decode step (k_decode_step.cu): its layer table, scratch,
  // barrier counter and the per-step argmax words
  int decode_path = 0;                   // B2A_DECODE_LAYERED or B2A_DECODE_PERSISTENT
  int step_ctas = 0;                     // 0: the step kernel does not fit this shape
  void* d_step = nullptr;
  b2a::StepLayer* step_layers = nullptr;
  float *sx = nullptr, *sqkv = nullptr, *spart = nullptr, *sh = nullptr;
  unsigned* bar = nullptr;
  int* abort_flag = nullptr;
  unsigned long long* keys = nullptr;    // [capacity + 1]
  unsigned bar_base = 0;
  int part_chunks = 0;                   // attention chunks per head the partials hold
};

using namespace b2a;

namespace {

size_t align256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

class ModelGuard {
 public:
  explicit ModelGuard(b2a_ctx* ctx) : ctx_(ctx), ok_(ctx_acquire(ctx)) {}
  ~ModelGuard() {
    if (ok_) ctx_release(ctx_);
  }
  bool ok() const { return ok_; }

 private:
  b2a_ctx* ctx_;
  bool ok_;
};

// Device or host source -> device destination, on the context's stream.
b2a_status copy_in(b2a_model* m, void* dst, const void* src, size_t bytes, int flags, const char* what) {
  if (src == nullptr) return fail(B2A_EINVAL, "null %s", what);
  const cudaMemcpyKind kind = flags == B2A_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
  const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, kind, m->ctx->stream);
  if (e != cudaSuccess) return cuda_fail(e, what);
  return B2A_OK;
}

// `rows` rows of `width` bytes, packed at the source, to every dst_pitch bytes.
b2a_status copy_rows(b2a_model* m, void* dst, size_t dst_pitch, const void* src, size_t width, size_t rows, int flags,
                     const char* what) {
  if (src == nullptr) return fail(B2A_EINVAL, "null %s", what);
  const cudaMemcpyKind kind = flags == B2A_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
  const cudaError_t e = cudaMemcpy2DAsync(dst, dst_pitch, src, width, width, rows, kind, m->ctx->stream);
  if (e != cudaSuccess) return cuda_fail(e, what);
  return B2A_OK;
}

b2a_status ensure_activations(b2a_model* m, int tokens) {
  if (tokens <= m->t_cap) return B2A_OK;
  const int t = std::max(tokens, 16);
  const b2a_model_config& c = m->cfg;
  const size_t h4 = align256(static_cast<size_t>(t) * c.hidden_size * 4);
  const size_t h2 = align256(static_cast<size_t>(t) * c.hidden_size * 2);
  const size_t kv2 = align256(static_cast<size_t>(t) * m->kv_dim * 2);
  const size_t i4 = align256(static_cast<size_t>(t) * c.intermediate_size * 4);
  const size_t total = 3 * h4 + h2 + 2 * kv2 + 3 * i4;
  if (m->d_act) {
    cudaError_t e = cudaFree(m->d_act);   // waits for work still using it
    m->d_act = nullptr;
    m->t_cap = 0;
    if (e != cudaSuccess) return cuda_fail(e, "freeing the activations");
  }
  cudaError_t e = cudaMalloc(&m->d_act, total);
  if (e != cudaSuccess) return cuda_fail(e, "allocating the activations");
  auto* p = static_cast<unsigned char*>(m->d_act);
  m->x = reinterpret_cast<float*>(p);
  m->nx = reinterpret_cast<float*>(p + h4);
  m->att = reinterpret_cast<float*>(p + 2 * h4);
  m->q = reinterpret_cast<uint16_t*>(p + 3 * h4);
  m->k = reinterpret_cast<uint16_t*>(p + 3 * h4 + h2);
  m->v = reinterpret_cast<uint16_t*>(p + 3 * h4 + h2 + kv2);
  m->gate = reinterpret_cast<float*>(p + 3 * h4 + h2 + 2 * kv2);
  m->up = reinterpret_cast<float*>(p + 3 * h4 + h2 + 2 * kv2 + 2 * i4);
  m->t_cap = t;
  return B2A_OK;
}

LinearParams linear(const int8_t* w, const void* s, int sdt, const float* bias, const void* x, int rows, int cols,
                    int tokens, void* out, int out_dtype, const void* residual) {
  LinearParams p{};
  p.w = w;
  p.scale = s;
  p.scale_dtype = sdt;
  p.bias = bias;
  p.bias_dtype = DT_F32;
  p.x = x;
  p.x_dtype = DT_F32;
  p.rows = rows;
  p.cols = cols;
  p.tokens = tokens;
  p.out[0] = out;
  p.seg_end[0] = rows;
  p.nseg = 1;
  p.out_dtype = out_dtype;
  p.residual = residual;
  return p;
}

#define MODEL_LAUNCH(kind, call, what)          \
  do {                                          \
    cudaError_t e_;                             \
    {                                           \
      KernelTimer kt_(ctx, kind);               \
      e_ = (call);                              \
    }                                           \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

// Before the first step kernel of a call: the barrier counter, the abort flag
// and the host's copy of the counter start from zero.
b2a_status step_reset(b2a_model* m) {
  if (m->bar == nullptr) return B2A_OK;
  const cudaError_t e = cudaMemsetAsync(m->bar, 0, 256, m->ctx->stream);   // counter and abort flag
  if (e != cudaSuccess) return cuda_fail(e, "resetting the step barrier");
  m->bar_base = 0;
  return B2A_OK;
}

bool step_fits(const b2a_model* m, int past) {
  const int chunk = decode_step_attn_chunk();
  return m->step_ctas > 0 && (past + chunk) / chunk <= m->part_chunks;
}

// One decode step of every layer in one cooperative launch: token *d_tok at
// the cache's length; the pick goes to *d_next (its logit to *d_best), the
// logits to m->logits; key_slot: a zeroed argmax word.
b2a_status run_step(b2a_model* m, const int32_t* d_tok, int32_t* d_next, float* d_best,
                    unsigned long long* key_slot) {
  b2a_ctx* ctx = m->ctx;
  const b2a_model_config& c = m->cfg;
  const int past = m->cache->len[0];
  StepParams p{};
  p.layers = m->step_layers;
  p.num_layers = c.num_layers;
  p.hidden = c.hidden_size;
  p.inter = c.intermediate_size;
  p.heads = c.num_heads;
  p.kv_heads = c.num_kv_heads;
  p.vocab = c.vocab_size;
  p.scale_dtype = c.scale_dtype == B2A_F32 ? DT_F32 : DT_F16;
  p.eps = c.rms_norm_eps;
  p.emb = m->emb;
  p.s_emb = m->s_emb;
  p.n_final = m->n_final;
  p.kc = static_cast<uint16_t*>(m->cache->d_k);
  p.vc = static_cast<uint16_t*>(m->cache->d_v);
  p.s_layer = m->cache->s_layer;
  p.s_head = m->cache->s_head;
  p.past = past;
  p.rope_cos = m->rope->d_cos;
  p.rope_sin = m->rope->d_sin;
  p.token_in = d_tok;
  p.token_out = d_next;
  p.best_out = d_best;
  p.key = key_slot;
  p.logits = m->logits;
  p.x = m->sx;
  p.qkv = m->sqkv;
  p.part = m->spart;
  p.h = m->sh;
  p.bar = m->bar;
  p.bar_base = m->bar_base;
  p.abort = m->abort_flag;
  p.err = ctx->d_err;
  p.len = m->cache->d_len;
  // attention items: every head x every chunk of decode_step_attn_chunk() keys
  p.attn_chunk = decode_step_attn_chunk();
  p.attn_nchunks = (past + p.attn_chunk) / p.attn_chunk;
  cudaError_t e;
  {
    KernelTimer kt(ctx, K_DECODE_STEP);
    e = launch_decode_step(p, m->step_ctas, ctx->stream);
  }
  if (e != cudaSuccess) return cuda_fail(e, "launching the decode step");
  m->bar_base += static_cast<unsigned>((decode_step_barriers(c.num_layers) + 1) * m->step_ctas);
  m->cache->len[0] += 1;   // the kernel set the device copy
  return B2A_OK;
}

// One forward over `count` tokens already on the device (d_tok), at the
// cache's length; leaves the last position's logits in m->logits and the
// argmax in *d_next (and its logit in *d_best when non-null). The caller has
// validated the shapes and holds the context.
b2a_status run_forward(b2a_model* m, const int32_t* d_tok, int count, int32_t* d_next, float* d_best,
                       unsigned long long* key_slot) {
  b2a_ctx* ctx = m->ctx;
  cudaStream_t st = ctx->stream;
  const b2a_model_config& c = m->cfg;
  const int H = c.hidden_size, I = c.intermediate_size, KV = m->kv_dim;
  const int sdt = c.scale_dtype == B2A_F32 ? DT_F32 : DT_F16;
  b2a_status s;
  if (count == 1 && key_slot != nullptr && m->decode_path == B2A_DECODE_PERSISTENT &&
      step_fits(m, m->cache->len[0])) {
    return run_step(m, d_tok, d_next, d_best, key_slot);
  }
  if ((s = ensure_activations(m, count)) != B2A_OK) return s;

  MODEL_LAUNCH(K_EMBED, launch_embed_int8(d_tok, count, m->emb, m->s_emb, sdt, H, c.vocab_size, m->x, ctx->d_err, st),
               "launching the embedding lookup");
  for (int l = 0; l < c.num_layers; l++) {
    const b2a_model::Layer& w = m->layers[l];
    // ---- attention block: src/cpu/model.js:98-128
    MODEL_LAUNCH(K_RMSNORM, launch_rmsnorm(m->x, w.n_in, c.rms_norm_eps, count, H, m->nx, st), "launching rmsnorm");
    LinearParams p = linear(w.qkv, w.s_qkv, sdt, w.b_qkv, m->nx, m->qkv_rows, H, count, m->q, DT_F16, nullptr);
    p.out[1] = m->k;
    p.out[2] = m->v;
    p.seg_end[0] = H;
    p.seg_end[1] = H + KV;
    p.seg_end[2] = H + 2 * KV;
    p.nseg = 3;
    MODEL_LAUNCH(K_LINEAR, launch_linear_int8(p, st), "launching the qkv projection");
    if (count == 1) {
      s = attn_decode_device(ctx, m->cache, m->rope, l, c.num_heads, m->q, m->k, m->v, B2A_F16, m->att, B2A_F32);
    } else {
      s = attn_prefill_device(ctx, m->cache, m->rope, l, 0, c.num_heads, m->q, m->k, m->v, B2A_F16, count, m->att,
                              B2A_F32);
    }
    if (s != B2A_OK) return s;
    p = linear(w.o, w.s_o, sdt, nullptr, m->att, H, H, count, m->x, DT_F32, m->x);
    MODEL_LAUNCH(K_LINEAR, launch_linear_int8(p, st), "launching the o projection");
    // ---- feed-forward: src/cpu/model.js:131-140
    MODEL_LAUNCH(K_RMSNORM, launch_rmsnorm(m->x, w.n_post, c.rms_norm_eps, count, H, m->nx, st),
                 "launching rmsnorm");
    p = linear(w.gu, w.s_gu, sdt, nullptr, m->nx, 2 * I, H, count, m->gate, DT_F32, nullptr);
    MODEL_LAUNCH(K_LINEAR, launch_linear_int8(p, st), "launching the gate/up projection");
    MODEL_LAUNCH(K_SWIGLU, launch_swiglu(m->gate, m->up, static_cast<int64_t>(count) * I, st), "launching swiglu");
    p = linear(w.down, w.s_down, sdt, nullptr, m->up, H, I, count, m->x, DT_F32, m->x);
    MODEL_LAUNCH(K_LINEAR, launch_linear_int8(p, st), "launching the down projection");
  }
  // only now are the new positions visible (src/cpu/model.js:145-146)
  m->cache->len[0] += count;
  {
    const cudaError_t e = launch_lengths_update(m->cache->d_len, 0, 1, count, 0, st);
    if (e != cudaSuccess) return cuda_fail(e, "updating the cache length");
  }
  // final norm of the last position and the tied output projection
  // (src/cpu/model.js:151-157, 214-230)
  const float* last = m->x + static_cast<int64_t>(count - 1) * H;
  MODEL_LAUNCH(K_RMSNORM, launch_rmsnorm(last, m->n_final, c.rms_norm_eps, 1, H, m->nx, st), "launching rmsnorm");
  LinearParams p = linear(m->emb, m->s_emb, sdt, nullptr, m->nx, c.vocab_size, H, 1, m->logits, DT_F32, nullptr);
  MODEL_LAUNCH(K_LINEAR, launch_linear_int8(p, st), "launching the output projection");
  MODEL_LAUNCH(K_ARGMAX, launch_argmax(m->logits, c.vocab_size, d_next, d_best, m->arg_scratch, st),
               "launching the argmax");
  return B2A_OK;
}

b2a_status check_loaded(const b2a_model* m) {
  for (int l = 0; l < m->cfg.num_layers; l++) {
    if (!m->layers[l].loaded) return fail(B2A_EINVAL, "weights of layer %d are not loaded", l);
  }
  if (!m->emb_loaded) return fail(B2A_EINVAL, "the embedding is not loaded");
  if (!m->final_loaded) return fail(B2A_EINVAL, "the final norm is not loaded");
  return B2A_OK;
}

// src/gpu/model.js:249-254
b2a_status check_room(const b2a_model* m, int count) {
  const int past = m->cache->len[0];
  if (static_cast<int64_t>(past) + count > m->capacity) {
    return fail(B2A_ERANGE, "cache holds %d of %d; cannot add %d", past, m->capacity, count);
  }
  if (static_cast<int64_t>(past) + count > m->cfg.max_positions) {
    return fail(B2A_ERANGE, "position %d exceeds the %d-entry rope table", past + count, m->cfg.max_positions);
  }
  return B2A_OK;
}

// src/cpu/model.js:200-203
b2a_status check_tokens(const b2a_model* m, const int32_t* ids, int n) {
  for (int t = 0; t < n; t++) {
    if (ids[t] < 0 || ids[t] >= m->cfg.vocab_size) {
      return fail(B2A_ERANGE, "token %d at position %d is outside the vocabulary", ids[t], t);
    }
  }
  return B2A_OK;
}

void free_model(b2a_model* m) {
  if (m == nullptr) return;
  cudaSetDevice(m->device);
  if (m->d_weights) cudaFree(m->d_weights);
  if (m->d_act) cudaFree(m->d_act);
  if (m->d_fixed) cudaFree(m->d_fixed);
  if (m->d_step) cudaFree(m->d_step);
  if (m->cache) b2a_kvcache_destroy(m->cache);
  if (m->rope) b2a_rope_destroy(m->rope);
  delete m;
}

}  // namespace

extern "C" {

b2a_status b2a_model_create(b2a_ctx* ctx, const b2a_model_config* cfg, int capacity, b2a_model** out) {
  if (out == nullptr || cfg == nullptr || ctx == nullptr) return fail(B2A_EINVAL, "null argument");
  *out = nullptr;
  const b2a_model_config& c = *cfg;
  // src/core/config.js:18-66
  if (c.num_heads < 1 || c.num_kv_heads < 1 || c.num_layers < 1 || c.vocab_size < 1 || c.intermediate_size < 16) {
    return fail(B2A_EINVAL, "config: bad sizes (heads %d/%d, layers %d, vocab %d, intermediate %d)", c.num_heads,
                c.num_kv_heads, c.num_layers, c.vocab_size, c.intermediate_size);
  }
  if (c.hidden_size % c.num_heads != 0) {
    return fail(B2A_EINVAL, "config: hidden_size %d is not divisible by num_attention_heads %d", c.hidden_size,
                c.num_heads);
  }
  if (c.num_heads % c.num_kv_heads != 0) {
    return fail(B2A_EINVAL,
                "config: num_attention_heads %d is not divisible by num_key_value_heads %d, so the query heads "
                "cannot be grouped evenly over the key/value heads",
                c.num_heads, c.num_kv_heads);
  }
  if (c.hidden_size / c.num_heads != 64) {
    return fail(B2A_EINVAL, "config: the attention kernels are built for head_dim 64, got %d",
                c.hidden_size / c.num_heads);
  }
  if (c.num_heads / c.num_kv_heads > 8) {
    return fail(B2A_EINVAL, "config: at most 8 query heads per KV head, got %d", c.num_heads / c.num_kv_heads);
  }
  if (c.intermediate_size % 16 != 0) {
    return fail(B2A_EINVAL, "config: intermediate_size %d must be a multiple of 16", c.intermediate_size);
  }
  if (!(c.rms_norm_eps >= 0) || !(c.rope_theta > 0) || c.max_positions < 1) {
    return fail(B2A_EINVAL, "config: bad rms_norm_eps, rope_theta or max_position_embeddings");
  }
  if (c.scale_dtype != B2A_F16 && c.scale_dtype != B2A_F32) return fail(B2A_EINVAL, "config: scales are f16 or f32");
  if (capacity < 1) return fail(B2A_ERANGE, "cache capacity must be a positive integer, got %d", capacity);

  b2a_model* m = new (std::nothrow) b2a_model();
  if (m == nullptr) return fail(B2A_EINVAL, "out of host memory");
  m->ctx = ctx;
  m->device = ctx->device;
  m->cfg = c;
  m->capacity = capacity;
  m->kv_dim = c.num_kv_heads * 64;
  m->qkv_rows = c.hidden_size + 2 * m->kv_dim;
  m->ssz = c.scale_dtype == B2A_F32 ? 4 : 2;
  b2a_status s = b2a_kvcache_create(ctx, c.num_layers, c.num_kv_heads, 64, capacity, 1, B2A_F16, &m->cache);
  if (s == B2A_OK) s = b2a_rope_create(ctx, 64, c.rope_theta, c.max_positions, &m->rope);
  if (s != B2A_OK) {
    free_model(m);
    return s;
  }
  ModelGuard g(ctx);
  if (!g.ok()) {
    free_model(m);
    return busy_fail(ctx);
  }
  const size_t H = c.hidden_size, I = c.intermediate_size, V = c.vocab_size, Q = m->qkv_rows;
  const size_t per_layer = align256(Q * H) + align256(H * H) + align256(2 * I * H) + align256(H * I) +
                           align256(Q * m->ssz) + align256(H * m->ssz) + align256(2 * I * m->ssz) +
                           align256(H * m->ssz) + align256(Q * 4) + 2 * align256(H * 4);
  const size_t total = per_layer * c.num_layers + align256(V * H) + align256(V * m->ssz) + align256(H * 4);
  cudaError_t e = cudaMalloc(&m->d_weights, total);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->d_weights, 0, total, ctx->stream);
  const size_t fixed = align256(V * 4) + 2 * align256(static_cast<size_t>(capacity) * 4) +
                       align256(static_cast<size_t>(capacity) * 4) + kArgmaxScratchBytes;
  if (e == cudaSuccess) e = cudaMalloc(&m->d_fixed, fixed);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->d_fixed, 0, fixed, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    free_model(m);
    return cuda_fail(e, "allocating the model");
  }
  auto* p = static_cast<unsigned char*>(m->d_weights);
  auto take = [&p](size_t bytes) {
    unsigned char* r = p;
    p += align256(bytes);
    return r;
  };
  m->layers.resize(c.num_layers);
  for (auto& L : m->layers) {
    L.qkv = reinterpret_cast<int8_t*>(take(Q * H));
    L.o = reinterpret_cast<int8_t*>(take(H * H));
    L.gu = reinterpret_cast<int8_t*>(take(2 * I * H));
    L.down = reinterpret_cast<int8_t*>(take(H * I));
    L.s_qkv = take(Q * m->ssz);
    L.s_o = take(H * m->ssz);
    L.s_gu = take(2 * I * m->ssz);
    L.s_down = take(H * m->ssz);
    L.b_qkv = reinterpret_cast<float*>(take(Q * 4));
    L.n_in = reinterpret_cast<float*>(take(H * 4));
    L.n_post = reinterpret_cast<float*>(take(H * 4));
    L.loaded = false;
  }
  m->emb = reinterpret_cast<int8_t*>(take(V * H));
  m->s_emb = take(V * m->ssz);
  m->n_final = reinterpret_cast<float*>(take(H * 4));
  auto* f = static_cast<unsigned char*>(m->d_fixed);
  m->logits = reinterpret_cast<float*>(f);
  f += align256(V * 4);
  m->tokens = reinterpret_cast<int32_t*>(f);
  f += align256(static_cast<size_t>(capacity) * 4);
  m->gen = reinterpret_cast<int32_t*>(f);
  f += align256(static_cast<size_t>(capacity) * 4);
  m->best = reinterpret_cast<float*>(f);
  f += align256(static_cast<size_t>(capacity) * 4);
  m->arg_scratch = f;

  // the one-kernel decode step, when this shape fits it
  const int ctas = decode_step_max_ctas();
  if (decode_step_supported(c.hidden_size, c.intermediate_size, m->qkv_rows, c.vocab_size, ctas)) {
    const int part_chunks = (capacity + decode_step_attn_chunk() - 1) / decode_step_attn_chunk();
    const size_t bytes = align256(sizeof(StepLayer) * c.num_layers) + align256(H * 4) + align256(Q * 4) +
                         align256(static_cast<size_t>(c.num_heads) * part_chunks * 68 * 4) + align256(I * 4) + 256 +
                         align256(sizeof(unsigned long long) * (static_cast<size_t>(capacity) + 1));
    e = cudaMalloc(&m->d_step, bytes);
    if (e == cudaSuccess) e = cudaMemsetAsync(m->d_step, 0, bytes, ctx->stream);
    std::vector<StepLayer> table(c.num_layers);
    for (int l = 0; l < c.num_layers; l++) {
      const b2a_model::Layer& L = m->layers[l];
      table[l] = StepLayer{L.qkv, L.o, L.gu, L.down, L.s_qkv, L.s_o, L.s_gu, L.s_down, L.b_qkv, L.n_in, L.n_post};
    }
    auto* q = static_cast<unsigned char*>(m->d_step);
    if (e == cudaSuccess) {
      e = cudaMemcpyAsync(q, table.data(), sizeof(StepLayer) * c.num_layers, cudaMemcpyHostToDevice, ctx->stream);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
      free_model(m);
      return cuda_fail(e, "allocating the decode-step state");
    }
    m->step_layers = reinterpret_cast<StepLayer*>(q);
    q += align256(sizeof(StepLayer) * c.num_layers);
    m->sx = reinterpret_cast<float*>(q);
    q += align256(H * 4);
    m->sqkv = reinterpret_cast<float*>(q);
    q += align256(Q * 4);
    m->spart = reinterpret_cast<float*>(q);
    q += align256(static_cast<size_t>(c.num_heads) * part_chunks * 68 * 4);
    m->sh = reinterpret_cast<float*>(q);
    q += align256(I * 4);
    m->bar = reinterpret_cast<unsigned*>(q);
    m->abort_flag = reinterpret_cast<int*>(q + 128);
    q += 256;
    m->keys = reinterpret_cast<unsigned long long*>(q);
    m->step_ctas = ctas;
    m->part_chunks = part_chunks;
    m->decode_path = B2A_DECODE_PERSISTENT;
  }
  *out = m;
  return B2A_OK;
}

b2a_status b2a_model_destroy(b2a_model* model) {
  free_model(model);
  return B2A_OK;
}

b2a_status b2a_model_load_layer(b2a_model* m, int layer, const b2a_layer_weights* w, int flags) {
  if (m == nullptr || w == nullptr) return fail(B2A_EINVAL, "null argument");
  if (layer < 0 || layer >= m->cfg.num_layers) {
    return fail(B2A_EINVAL, "layer %d out of range [0, %d)", layer, m->cfg.num_layers);
  }
  ModelGuard g(m->ctx);
  if (!g.ok()) return busy_fail(m->ctx);
  const size_t H = m->cfg.hidden_size, I = m->cfg.intermediate_size, Q = m->qkv_rows, ss = m->ssz;
  b2a_model::Layer& L = m->layers[layer];
  b2a_status s;
  if ((s = copy_in(m, L.n_in, w->input_norm, H * 4, flags, "input_norm")) != B2A_OK) return s;
  if ((s = copy_in(m, L.n_post, w->post_attn_norm, H * 4, flags, "post_attn_norm")) != B2A_OK) return s;
  if ((s = copy_in(m, L.qkv, w->qkv, Q * H, flags, "qkv codes")) != B2A_OK) return s;
  if ((s = copy_in(m, L.s_qkv, w->qkv_scales, Q * ss, flags, "qkv scales")) != B2A_OK) return s;
  if ((s = copy_in(m, L.b_qkv, w->qkv_bias, Q * 4, flags, "qkv bias")) != B2A_OK) return s;
  if ((s = copy_in(m, L.o, w->o, H * H, flags, "o codes")) != B2A_OK) return s;
  if ((s = copy_in(m, L.s_o, w->o_scales, H * ss, flags, "o scales")) != B2A_OK) return s;
  // gate row i -> row 2i, up row i -> row 2i + 1 (and the same for the scales)
  if ((s = copy_rows(m, L.gu, 2 * H, w->gate, H, I, flags, "gate codes")) != B2A_OK) return s;
  if ((s = copy_rows(m, L.gu + H, 2 * H, w->up, H, I, flags, "up codes")) != B2A_OK) return s;
  if ((s = copy_rows(m, L.s_gu, 2 * ss, w->gate_scales, ss, I, flags, "gate scales")) != B2A_OK) return s;
  if ((s = copy_rows(m, static_cast<unsigned char*>(L.s_gu) + ss, 2 * ss, w->up_scales, ss, I, flags,
                     "up scales")) != B2A_OK) {
    return s;
  }
  if ((s = copy_in(m, L.down, w->down, H * I, flags, "down codes")) != B2A_OK) return s;
  if ((s = copy_in(m, L.s_down, w->down_scales, H * ss, flags, "down scales")) != B2A_OK) return s;
  if ((s = stream_sync_check(m->ctx)) != B2A_OK) return s;
  L.loaded = true;
  return B2A_OK;
}

b2a_status b2a_model_load_embedding(b2a_model* m, const int8_t* codes, const void* scales, int flags) {
  if (m == nullptr) return fail(B2A_EINVAL, "null model");
  ModelGuard g(m->ctx);
  if (!g.ok()) return busy_fail(m->ctx);
  const size_t H = m->cfg.hidden_size, V = m->cfg.vocab_size;
  b2a_status s;
  if ((s = copy_in(m, m->emb, codes, V * H, flags, "embedding codes")) != B2A_OK) return s;
  if ((s = copy_in(m, m->s_emb, scales, V * m->ssz, flags, "embedding scales")) != B2A_OK) return s;
  if ((s = stream_sync_check(m->ctx)) != B2A_OK) return s;
  m->emb_loaded = true;
  return B2A_OK;
}

b2a_status b2a_model_load_final_norm(b2a_model* m, const float* weight, int flags) {
  if (m == nullptr) return fail(B2A_EINVAL, "null model");
  ModelGuard g(m->ctx);
  if (!g.ok()) return busy_fail(m->ctx);
  b2a_status s = copy_in(m, m->n_final, weight, static_cast<size_t>(m->cfg.hidden_size) * 4, flags, "final norm");
  if (s == B2A_OK) s = stream_sync_check(m->ctx);
  if (s == B2A_OK) m->final_loaded = true;
  return s;
}

b2a_status b2a_model_forward(b2a_model* m, const int32_t* tokens, int seq, float* logits, int32_t* next_token,
                             int flags) {
  if (m == nullptr) return fail(B2A_EINVAL, "null model");
  if (seq < 1) return fail(B2A_EINVAL, "forward: need at least one token");
  if (tokens == nullptr) return fail(B2A_EINVAL, "null tokens");
  b2a_status s;
  if ((s = check_loaded(m)) != B2A_OK) return s;
  if ((s = check_room(m, seq)) != B2A_OK) return s;
  if (flags == B2A_HOST && (s = check_tokens(m, tokens, seq)) != B2A_OK) return s;
  ModelGuard g(m->ctx);
  if (!g.ok()) return busy_fail(m->ctx);
  cudaStream_t st = m->ctx->stream;
  const int32_t* d_tok = tokens;
  int32_t* d_next = next_token;
  if (flags == B2A_HOST) {
    cudaError_t e = cudaMemcpyAsync(m->tokens, tokens, sizeof(int32_t) * seq, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "copying tokens to the device");
    d_tok = m->tokens;
    d_next = m->gen;
  } else if (d_next == nullptr) {
    d_next = m->gen;
  }
  if ((s = step_reset(m)) != B2A_OK) return s;
  if (m->keys) {
    cudaError_t e = cudaMemsetAsync(m->keys, 0, sizeof(unsigned long long), st);
    if (e != cudaSuccess) return cuda_fail(e, "clearing the argmax word");
  }
  if ((s = run_forward(m, d_tok, seq, d_next, nullptr, m->keys)) != B2A_OK) return s;
  const size_t lbytes = static_cast<size_t>(m->cfg.vocab_size) * 4;
  if (flags == B2A_HOST) {
    cudaError_t e = cudaSuccess;
    if (logits) e = cudaMemcpyAsync(logits, m->logits, lbytes, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && next_token) e = cudaMemcpyAsync(next_token, d_next, 4, cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return cuda_fail(e, "copying results to the host");
    return stream_sync_check(m->ctx);
  }
  if (logits) {
    cudaError_t e = cudaMemcpyAsync(logits, m->logits, lbytes, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "copying the logits");
  }
  return B2A_OK;
}

b2a_status b2a_model_generate(b2a_model* m, const int32_t* prompt, int n_prompt, int max_tokens,
                              const int32_t* stop_tokens, int n_stop, int32_t* tokens_out, float* best_logits,
                              int* n_generated) {
  if (m == nullptr || prompt == nullptr || tokens_out == nullptr || n_generated == nullptr) {
    return fail(B2A_EINVAL, "null argument");
  }
  *n_generated = 0;
  if (n_prompt < 1) return fail(B2A_EINVAL, "forward: need at least one token");
  if (max_tokens < 0 || n_stop < 0 || (n_stop > 0 && stop_tokens == nullptr)) {
    return fail(B2A_EINVAL, "bad max_tokens or stop tokens");
  }
  if (max_tokens == 0) return B2A_OK;
  b2a_status s;
  if ((s = check_loaded(m)) != B2A_OK) return s;
  if ((s = check_tokens(m, prompt, n_prompt)) != B2A_OK) return s;
  // a fresh cache (src/cpu/model.js:167): the prompt, then every generated
  // token but the last is run
  const int need = n_prompt + max_tokens - 1;
  if (need > m->capacity) return fail(B2A_ERANGE, "cache holds 0 of %d; cannot add %d", m->capacity, need);
  if (need > m->cfg.max_positions) {
    return fail(B2A_ERANGE, "position %d exceeds the %d-entry rope table", need, m->cfg.max_positions);
  }
  ModelGuard g(m->ctx);
  if (!g.ok()) return busy_fail(m->ctx);
  cudaStream_t st = m->ctx->stream;
  m->cache->len[0] = 0;
  cudaError_t e = launch_lengths_update(m->cache->d_len, 0, 1, 0, 1, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(m->tokens, prompt, sizeof(int32_t) * n_prompt, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && m->keys) {
    e = cudaMemsetAsync(m->keys, 0, sizeof(unsigned long long) * (m->capacity + 1), st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "starting the generation");
  if ((s = step_reset(m)) != B2A_OK) return s;
  int done = 0;
  for (int step = 0; step < max_tokens; step++) {
    const int32_t* in = step == 0 ? m->tokens : m->gen + step - 1;
    if ((s = run_forward(m, in, step == 0 ? n_prompt : 1, m->gen + step, m->best + step,
                         m->keys ? m->keys + step : nullptr)) != B2A_OK) {
      return s;
    }
    done = step + 1;
    if (n_stop > 0) {   // the host sees each token before deciding to go on
      int32_t tok = 0;
      e = cudaMemcpyAsync(&tok, m->gen + step, 4, cudaMemcpyDeviceToHost, st);
      if (e != cudaSuccess) return cuda_fail(e, "reading the generated token");
      if ((s = stream_sync_check(m->ctx)) != B2A_OK) return s;
      if (std::find(stop_tokens, stop_tokens + n_stop, tok) != stop_tokens + n_stop) break;
    }
  }
  e = cudaMemcpyAsync(tokens_out, m->gen, sizeof(int32_t) * done, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess && best_logits) {
    e = cudaMemcpyAsync(best_logits, m->best, sizeof(float) * done, cudaMemcpyDeviceToHost, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "copying the generated tokens");
  if ((s = stream_sync_check(m->ctx)) != B2A_OK) return s;
  *n_generated = done;
  return B2A_OK;
}

b2a_status b2a_model_set_decode_path(b2a_model* m, int path) {
  if (m == nullptr) return fail(B2A_EINVAL, "null model");
  if (path != B2A_DECODE_LAYERED && path != B2A_DECODE_PERSISTENT) return fail(B2A_EINVAL, "unknown decode path %d", path);
  if (path == B2A_DECODE_PERSISTENT && m->step_ctas <= 0) {
    return fail(B2A_EINVAL, "this model's shape does not fit the one-kernel decode step");
  }
  m->decode_path = path;
  return B2A_OK;
}

b2a_status b2a_model_decode_path(const b2a_model* m, int* path) {
  if (m == nullptr || path == nullptr) return fail(B2A_EINVAL, "null argument");
  *path = m->decode_path;
  return B2A_OK;
}

b2a_status b2a_model_reset(b2a_model* m) {
  if (m == nullptr) return fail(B2A_EINVAL, "null model");
  return b2a_kvcache_reset(m->cache, 0);
}

b2a_status b2a_model_length(const b2a_model* m, int* length) {
  if (m == nullptr || length == nullptr) return fail(B2A_EINVAL, "null argument");
  *length = m->cache->len[0];
  return B2A_OK;
}

b2a_status b2a_model_cache(b2a_model* m, b2a_kvcache** cache) {
  if (m == nullptr || cache == nullptr) return fail(B2A_EINVAL, "null argument");
  *cache = m->cache;
  return B2A_OK;
}

}  // extern "C"

// ---------------------------------------------------------- weights from a file --

namespace {

// f32 -> f16 bits, round to nearest even (what a Float16 store does)
uint16_t host_f32_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return static_cast<uint16_t>(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u | ((ax >> 13) & 0x3ffu) : 0u));
  if (ax >= 0x477ff000u) return static_cast<uint16_t>(sign | 0x7c00u);   // rounds to infinity
  if (ax < 0x38800000u) {                                               // f16 subnormal or zero
    float a;
    std::memcpy(&a, &ax, 4);
    return static_cast<uint16_t>(sign | static_cast<uint32_t>(std::nearbyint(a * 16777216.0f)));
  }
  uint32_t h = (((ax >> 23) - 112u) << 10) | ((ax & 0x7fffffu) >> 13);
  const uint32_t rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return static_cast<uint16_t>(sign | h);
}

std::string shape_text(const std::vector<int64_t>& s) {
  std::string t;
  for (size_t k = 0; k < s.size(); k++) t += (k ? "," : "") + std::to_string(s[k]);
  return t;
}

// rows x cols of tensor `name` from row r0: widened to f32, quantized per row
// (quantize.js:36-58), codes to `codes`, scales (in the model's dtype) to `scales`.
b2a_status quantize_rows(const b2a_model* m, const b2a_safetensors* st, const char* name, int64_t r0, int rows,
                         int cols, int8_t* codes, unsigned char* scales, std::vector<float>& f,
                         std::vector<float>& s32) {
  char dt[16];
  b2a_status s = b2a_safetensors_info(st, name, dt, nullptr, 0, nullptr, nullptr);
  if (s != B2A_OK) return s;
  int64_t bytes = 0;
  b2a_safetensors_info(st, name, nullptr, nullptr, 0, nullptr, &bytes);
  int esz = std::string(dt) == "F64" ? 8 : (std::string(dt) == "F32" ? 4 : 2);
  const size_t n = static_cast<size_t>(rows) * cols;
  std::vector<unsigned char> raw(n * esz);
  f.resize(n);
  s32.resize(rows);
  if ((s = st_read_range(st, name, static_cast<uint64_t>(r0) * cols * esz, n * esz, raw.data())) != B2A_OK) return s;
  if (!st_widen(dt, raw.data(), n, f.data())) return fail(B2A_EINVAL, "%s: cannot widen %s to f32", name, dt);
  if ((s = b2a_quantize_int8_per_channel(f.data(), rows, cols, codes, s32.data())) != B2A_OK) return s;
  for (int r = 0; r < rows; r++) {
    if (m->ssz == 4) {
      std::memcpy(scales + 4 * r, &s32[r], 4);
    } else {
      const uint16_t h = host_f32_to_f16(s32[r]);
      std::memcpy(scales + 2 * r, &h, 2);
    }
  }
  return B2A_OK;
}

b2a_status read_vector(const b2a_safetensors* st, const std::string& name, float* dst, size_t n) {
  return b2a_safetensors_read_f32(st, name.c_str(), dst, n);
}

}  // namespace

extern "C" b2a_status b2a_model_load_safetensors(b2a_model* m, const b2a_safetensors* st) {
  if (m == nullptr || st == nullptr) return fail(B2A_EINVAL, "null argument");
  const b2a_model_config& c = m->cfg;
  const int64_t H = c.hidden_size, I = c.intermediate_size, KV = m->kv_dim, V = c.vocab_size;
  // config.expectedTensors / checkAgainst (src/core/config.js:88-150), tied embeddings
  std::vector<std::pair<std::string, std::vector<int64_t>>> want;
  want.push_back({"model.embed_tokens.weight", {V, H}});
  want.push_back({"model.norm.weight", {H}});
  for (int l = 0; l < c.num_layers; l++) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    want.push_back({p + "input_layernorm.weight", {H}});
    want.push_back({p + "post_attention_layernorm.weight", {H}});
    want.push_back({p + "self_attn.q_proj.weight", {H, H}});
    want.push_back({p + "self_attn.q_proj.bias", {H}});
    want.push_back({p + "self_attn.k_proj.weight", {KV, H}});
    want.push_back({p + "self_attn.k_proj.bias", {KV}});
    want.push_back({p + "self_attn.v_proj.weight", {KV, H}});
    want.push_back({p + "self_attn.v_proj.bias", {KV}});
    want.push_back({p + "self_attn.o_proj.weight", {H, H}});
    want.push_back({p + "mlp.gate_proj.weight", {I, H}});
    want.push_back({p + "mlp.up_proj.weight", {I, H}});
    want.push_back({p + "mlp.down_proj.weight", {H, I}});
  }
  std::vector<std::string> problems;
  for (const auto& e : want) {
    int64_t shape[8];
    int nd = 0;
    if (b2a_safetensors_info(st, e.first.c_str(), nullptr, shape, 8, &nd, nullptr) != B2A_OK) {
      problems.push_back("missing " + e.first);
      continue;
    }
    const std::vector<int64_t> got(shape, shape + std::min(nd, 8));
    if (got != e.second) {
      problems.push_back(e.first + ": expected shape [" + shape_text(e.second) + "], file has [" + shape_text(got) +
                         "]");
    }
  }
  for (int i = 0; i < b2a_safetensors_count(st); i++) {
    const std::string name = b2a_safetensors_name(st, i);
    bool known = false;
    for (const auto& e : want) known |= e.first == name;
    if (!known) problems.push_back("unexpected tensor " + name);
  }
  if (!problems.empty()) {
    std::string msg = "weights do not match config (" + std::to_string(problems.size()) + " problem" +
                      (problems.size() == 1 ? "" : "s") + "):";
    for (size_t k = 0; k < problems.size() && k < 10; k++) msg += "\n  " + problems[k];
    if (problems.size() > 10) msg += "\n  ... and " + std::to_string(problems.size() - 10) + " more";
    return fail(B2A_EINVAL, "%s", msg.c_str());
  }

  const int64_t Q = m->qkv_rows;
  const size_t ss = m->ssz;
  std::vector<float> f, s32;
  b2a_status s;
  for (int l = 0; l < c.num_layers; l++) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    std::vector<int8_t> qkv(Q * H), o(H * H), gate(I * H), up(I * H), down(H * I);
    std::vector<unsigned char> sqkv(Q * ss), so(H * ss), sg(I * ss), su(I * ss), sd(H * ss);
    std::vector<float> bias(Q), nin(H), npost(H);
    if ((s = quantize_rows(m, st, (p + "self_attn.q_proj.weight").c_str(), 0, H, H, qkv.data(), sqkv.data(), f, s32)) ||
        (s = quantize_rows(m, st, (p + "self_attn.k_proj.weight").c_str(), 0, KV, H, qkv.data() + H * H,
                           sqkv.data() + H * ss, f, s32)) ||
        (s = quantize_rows(m, st, (p + "self_attn.v_proj.weight").c_str(), 0, KV, H, qkv.data() + (H + KV) * H,
                           sqkv.data() + (H + KV) * ss, f, s32)) ||
        (s = quantize_rows(m, st, (p + "self_attn.o_proj.weight").c_str(), 0, H, H, o.data(), so.data(), f, s32)) ||
        (s = quantize_rows(m, st, (p + "mlp.gate_proj.weight").c_str(), 0, I, H, gate.data(), sg.data(), f, s32)) ||
        (s = quantize_rows(m, st, (p + "mlp.up_proj.weight").c_str(), 0, I, H, up.data(), su.data(), f, s32)) ||
        (s = quantize_rows(m, st, (p + "mlp.down_proj.weight").c_str(), 0, H, I, down.data(), sd.data(), f, s32)) ||
        (s = read_vector(st, p + "self_attn.q_proj.bias", bias.data(), H)) ||
        (s = read_vector(st, p + "self_attn.k_proj.bias", bias.data() + H, KV)) ||
        (s = read_vector(st, p + "self_attn.v_proj.bias", bias.data() + H + KV, KV)) ||
        (s = read_vector(st, p + "input_layernorm.weight", nin.data(), H)) ||
        (s = read_vector(st, p + "post_attention_layernorm.weight", npost.data(), H))) {
      return s;
    }
    b2a_layer_weights w{nin.data(), npost.data(), qkv.data(), sqkv.data(), bias.data(), o.data(), so.data(),
                        gate.data(), sg.data(), up.data(), su.data(), down.data(), sd.data()};
    if ((s = b2a_model_load_layer(m, l, &w, B2A_HOST)) != B2A_OK) return s;
  }
  // the embedding in blocks of rows (272 MB of bfloat16 for Qwen2.5-0.5B)
  std::vector<int8_t> ecodes(V * H);
  std::vector<unsigned char> escales(V * ss);
  constexpr int64_t kBlock = 8192;
  for (int64_t r = 0; r < V; r += kBlock) {
    const int rows = static_cast<int>(std::min(kBlock, V - r));
    if ((s = quantize_rows(m, st, "model.embed_tokens.weight", r, rows, static_cast<int>(H), ecodes.data() + r * H,
                           escales.data() + r * ss, f, s32)) != B2A_OK) {
      return s;
    }
  }
  if ((s = b2a_model_load_embedding(m, ecodes.data(), escales.data(), B2A_HOST)) != B2A_OK) return s;
  std::vector<float> fin(H);
  if ((s = read_vector(st, "model.norm.weight", fin.data(), H)) != B2A_OK) return s;
  return b2a_model_load_final_norm(m, fin.data(), B2A_HOST);
}
