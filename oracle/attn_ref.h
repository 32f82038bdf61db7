/*
 * attn_ref.h -- CPU restatement of the reference engine's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity oracle for the CUDA
 * kernels in libb2a.so. Only the test suite, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py may load it, and only as the checker or as the
 * timed CPU baseline. The product path never calls it and has no CPU fallback.
 *
 * The reference (abho7/llm-inference-webgpu) is JavaScript. Its numeric
 * semantics are restated here exactly:
 *   - a JS number is an IEEE f64, so every accumulator below is a double;
 *   - a Float32Array store rounds to nearest-even f32, so every such store is
 *     an explicit (float) cast;
 *   - JS never contracts a*b+c into an FMA, so this file is compiled with
 *     -ffp-contract=off.
 * Math.exp / Math.cos / Math.sin / Math.pow are V8 builtins; this file uses
 * glibc's, which agree with them to within 1 ulp of f64 (far inside every
 * tolerance used), and which are the same functions the host uses to build
 * the f64 RoPE table the device reads, so the KV-cache bytes stay bit-exact.
 *
 * Parity pinning: the reference ships no numeric golden vectors for this path
 * that can be reproduced without the (absent) model weights. The restatement
 * is pinned by the reference's own known-answer and property tests
 * (test/attention.test.js, test/ops.test.js, test/cache.test.js,
 * test/dtype.test.js, web/kernels.html), restated in tests/ against this
 * library, and by an independent pure-Python transliteration of the JS
 * (tests/golden/make_golden.py) whose outputs are committed as fixtures.
 */
#ifndef B2A_ATTN_REF_H
#define B2A_ATTN_REF_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- dtype conversions: src/core/dtype.js ---------------------------------- */
float    or_bf16_to_f32(uint16_t bits);            /* dtype.js:17-20   */
uint16_t or_f32_to_bf16(float x);                  /* dtype.js:23-35   */
float    or_f16_to_f32(uint16_t bits);             /* dtype.js:55-78   */
uint16_t or_f32_to_f16(float x);                   /* dtype.js:81-113  */
void or_f32_to_f16_array(const float* src, uint16_t* dst, size_t n);
void or_f16_to_f32_array(const uint16_t* src, float* dst, size_t n);
void or_f32_to_bf16_array(const float* src, uint16_t* dst, size_t n);
void or_bf16_to_f32_array(const uint16_t* src, float* dst, size_t n);

/* ---- numeric ops: src/core/ops.js ----------------------------------------- */
void or_softmax_inplace(float* x, int n);                                   /* ops.js:66-78   */
void or_rope_frequencies(int head_dim, double theta, double* inv_freq);     /* ops.js:99-104  */
void or_rope_tables(int head_dim, double theta, int positions,
                    float* cos_out, float* sin_out);                        /* ops.js:123-136 */
/* The same angles kept in f64 (the table the device reads; see b2a_rope_create). */
void or_rope_tables_f64(int head_dim, double theta, int positions,
                        double* cos_out, double* sin_out);
void or_rope_inplace(float* vec, int offset, int head_dim, int position,
                     const double* inv_freq);                               /* ops.js:147-158 */

/* ---- attention: src/core/attention.js ------------------------------------- */
int  or_kv_head_for(int query_head, int num_heads, int num_kv_heads);       /* attention.js:74-76 */
void or_grouped_attention(const float* q, const float* keys, const float* values,
                          float* out, float* scores, int seq, int past,
                          int num_heads, int num_kv_heads, int head_dim);   /* attention.js:32-66 */
/* Multi-head attention over explicitly repeated KV heads: the comparison the
 * reference's own test builds (test/attention.test.js:15-58). */
void or_expanded_attention(const float* q, const float* keys, const float* values,
                           float* out, int seq, int past,
                           int num_heads, int num_kv_heads, int head_dim);

/* ---- KV cache: src/cpu/cache.js -------------------------------------------- */
typedef struct or_kvcache or_kvcache;
/* Returns NULL and fills err (if non-NULL) on a bad capacity (cache.js:23-26). */
or_kvcache* or_kvcache_new(int num_layers, int kv_dim, int capacity, char* err, size_t errlen);
void or_kvcache_free(or_kvcache* c);
int  or_kvcache_length(const or_kvcache* c);
int  or_kvcache_capacity(const or_kvcache* c);
size_t or_kvcache_byte_length(const or_kvcache* c);                         /* cache.js:41-43  */
/* Returns the start position, or -1 with err filled when it would overflow (cache.js:52-60). */
int  or_kvcache_allocate(or_kvcache* c, int count, char* err, size_t errlen);
void or_kvcache_write_at(or_kvcache* c, int layer, int at, const float* keys,
                         const float* values, int count);                   /* cache.js:63-67  */
const float* or_kvcache_keys_up_to(const or_kvcache* c, int layer, int n);  /* cache.js:75-77  */
const float* or_kvcache_values_up_to(const or_kvcache* c, int layer, int n);/* cache.js:79-81  */
void or_kvcache_commit(or_kvcache* c, int count);                           /* cache.js:84-86  */
void or_kvcache_present(const or_kvcache* c, int layer, int num_kv_heads, int head_dim,
                        float* key_out, float* value_out);                  /* cache.js:97-115 */
void or_kvcache_reset(or_kvcache* c);                                       /* cache.js:118    */

/* ---- one decoder layer's attention block: src/cpu/model.js:103-123 -------- */
/* RoPE on every query and KV head at absolute position past+t, append K/V,
 * attend over past+seq. q [seq, H*D] and k [seq, KVH*D] are rotated in place;
 * out [seq, H*D]. */
void or_layer_attention(or_kvcache* c, int layer, float* q, float* k, const float* v,
                        float* out, int seq, int num_heads, int num_kv_heads, int head_dim,
                        const double* inv_freq);

/* ---- batched decode and split-KV (the CUDA path's semantics, restated) ---- */
/* One new token per sequence over a head-major cache [kvh][pos][D] (the
 * layout KVCache.present() publishes, cache.js:97-115). The cache already
 * holds positions 0..len-1 and the new key/value at position len.
 * q [H*D] is already rotated; out [H*D]. Same arithmetic as
 * or_grouped_attention with seq=1, past=len. */
void or_decode_head_major(const float* q, const float* kcache, const float* vcache,
                          int cap, int len, int num_heads, int num_kv_heads,
                          int head_dim, float* out);
/* Partial (m, l, o) of one chunk [p0, p1) for one query head, in natural-log
 * units: m = max score, l = sum exp(s-m), o = sum exp(s-m) v (unnormalised). */
void or_decode_partial(const float* qh, const float* kh, const float* vh,
                       int p0, int p1, int head_dim, float* m, float* l, float* o);
/* Log-sum-exp combine of G partials in ascending order. */
void or_lse_combine(const float* m, const float* l, const float* o, int g,
                    int head_dim, float* out);

/* ---- seeded generators ----------------------------------------------------- */
/* The reference tests' uint32 LCG, values in [-1, 1] (test/attention.test.js:60-69). */
void or_random_array(float* out, size_t n, uint32_t seed);
/* Seeded N(0,1) for BASELINE's synthetic configs: splitmix64 -> Box-Muller. */
void or_normal_array(float* out, size_t n, uint64_t seed);

/* ---- multi-threaded batched decode (CPU baseline) -------------------------- */
/* For each (b, h): out[b*out_stride + h*D ..] = decode over positions
 * 0..len[b] inclusive of a head-major f16 cache whose sequence b starts at
 * b*seq_stride elements and is laid out [kvh][cap][D]; q[b*q_stride + h*D ..].
 * Widens f16 to f32 per element read, then the same arithmetic as
 * or_grouped_attention.
 * threads <= 0 uses every core. Returns the thread count used. */
int or_batched_decode_f16(const float* q, size_t q_stride, const uint16_t* kcache,
                          const uint16_t* vcache, size_t seq_stride, const int32_t* len,
                          int batch, int cap, int num_heads, int num_kv_heads, int head_dim,
                          float* out, size_t out_stride, int threads);


/* ---- projections (the layer's neighbours of attention) ---------------------- */
/* quantize.js:36-58: symmetric int8 per output row; scale = peak/127 stored as
 * f32, codes = roundHalfAwayFromZero(w / scale) (the division by the f64 scale)
 * clamped to [-127, 127]; an all-zero row gets scale 0 and zero codes. */
void or_quantize_int8_per_channel(const float* w, int rows, int cols, int8_t* codes, float* scales);
/* quantize.js:60-67: codes * scale, stored f32. */
void or_dequantize_int8_per_channel(const int8_t* codes, const float* scales, int rows, int cols, float* out);
/* ops.js:33-41: out[r] = bias[r] + sum_c W[r][c] x[c], f64 accumulation, f32 store. */
void or_matvec(const float* w, const float* x, int rows, int cols, const float* bias, float* out);

/* ---- the decoder around attention: src/core/ops.js, src/cpu/model.js ------- */
void   or_rmsnorm(const float* x, const float* weight, double eps, int n, float* out);  /* ops.js:17-24 */
double or_silu(double x);                                                             /* ops.js:81-83 */
void   or_swiglu_inplace(float* gate, const float* up, int n);                        /* ops.js:88-91 */
int    or_argmax(const float* logits, int n);                                         /* model.js:181-183 */
/* A Qwen2 decoder over int8 weights (one f32 scale per output row, the codes
 * widened per element as or_dequantize_int8_per_channel does) and its own f32
 * KV cache. The weight arrays are borrowed: the caller keeps them alive.
 * Matrix rows run on `threads` OpenMP threads. */
typedef struct or_model or_model;
or_model* or_model_new(int hidden, int inter, int layers, int heads, int kv_heads, int vocab, double theta,
                       double eps, int capacity, int threads);
void or_model_free(or_model* m);
/* qkv [hidden + 2 kv_dim][hidden] with q rows, k rows, v rows; o [hidden][hidden];
 * gate, up [inter][hidden]; down [hidden][inter]. */
void or_model_set_layer(or_model* m, int layer, const float* in_norm, const float* post_norm, const int8_t* qkv,
                        const float* qkv_scales, const float* qkv_bias, const int8_t* o, const float* o_scales,
                        const int8_t* gate, const float* gate_scales, const int8_t* up, const float* up_scales,
                        const int8_t* down, const float* down_scales);
void or_model_set_embedding(or_model* m, const int8_t* codes, const float* scales, const float* final_norm);
/* model.js:55-161 on the model's cache; returns the greedy pick or -1 (err). */
int  or_model_forward(or_model* m, const int32_t* tokens, int seq, float* logits_out, char* err, size_t errlen);
int  or_model_length(const or_model* m);
void or_model_reset(or_model* m);
/* cache.js:97-115: [kv_heads][length][head_dim] */
void or_model_present(const or_model* m, int layer, float* key_out, float* value_out);

#ifdef __cplusplus
}
#endif
#endif
