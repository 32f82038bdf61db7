/*
 * attn_ref.c -- CPU restatement of the reference engine's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see attn_ref.h): the parity oracle and the timed
 * CPU baseline, never part of the product path.
 *
 * Every function cites the reference file:line it restates. Compile with
 * -ffp-contract=off: JavaScript evaluates a*b+c as two rounded f64 operations.
 */
#include "attn_ref.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#if defined(__FP_FAST_FMA) && !defined(B2A_ALLOW_FMA)
/* Not an error by itself (the macro only says fma() is fast), but this file
 * must be built with -ffp-contract=off; the Makefile does that. */
#endif

static inline uint32_t f32_bits(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float bits_f32(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/* ---------------------------------------------------------------- dtype ---- */

/* src/core/dtype.js:17-20 -- bf16 is the top half of an f32. */
float or_bf16_to_f32(uint16_t bits) { return bits_f32((uint32_t)bits << 16); }

/* src/core/dtype.js:23-35 -- round to nearest even; NaN kept NaN with a quiet bit. */
uint16_t or_f32_to_bf16(float x) {
  uint32_t u = f32_bits(x);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu) != 0) {
    return (uint16_t)(((u >> 16) | 0x0040u) & 0xffffu);
  }
  uint32_t lsb = (u >> 16) & 1u;
  return (uint16_t)(((uint64_t)u + 0x7fffu + lsb) >> 16);
}

/* src/core/dtype.js:55-78 */
float or_f16_to_f32(uint16_t bits) {
  uint32_t sign = ((uint32_t)bits & 0x8000u) << 16;
  uint32_t exp = (bits >> 10) & 0x1fu;
  uint32_t mant = bits & 0x3ffu;
  uint32_t out;
  if (exp == 0x1f) {
    out = sign | 0x7f800000u | (mant << 13);
  } else if (exp == 0) {
    if (mant == 0) {
      out = sign;
    } else {
      int e = -1;
      uint32_t m = mant;
      do { m <<= 1; e++; } while ((m & 0x400u) == 0);
      out = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3ffu) << 13);
    }
  } else {
    out = sign | ((exp - 15 + 127) << 23) | (mant << 13);
  }
  return bits_f32(out);
}

/* src/core/dtype.js:81-113 -- RNE, overflow to inf, gradual underflow. */
uint16_t or_f32_to_f16(float x) {
  uint32_t u = f32_bits(x);
  uint32_t sign = (u >> 16) & 0x8000u;
  int exp = (int)((u >> 23) & 0xffu);
  uint32_t mant = u & 0x7fffffu;
  if (exp == 0xff) {
    return (uint16_t)(sign | 0x7c00u | (mant != 0 ? ((mant >> 13) | 0x200u) : 0u));
  }
  int e = exp - 127 + 15;
  if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    uint32_t m = mant | 0x800000u;
    int shift = 14 - e;
    uint32_t half = 1u << (shift - 1);
    uint32_t lsb = (m >> shift) & 1u;
    return (uint16_t)(sign | ((m + half - 1 + lsb) >> shift));
  }
  uint32_t lsb = (mant >> 13) & 1u;
  uint32_t rounded = mant + 0x0fffu + lsb;
  return (uint16_t)(sign | (((uint32_t)e << 10) + (rounded >> 13)));
}

void or_f32_to_f16_array(const float* src, uint16_t* dst, size_t n) {
  for (size_t i = 0; i < n; i++) dst[i] = or_f32_to_f16(src[i]);
}
void or_f16_to_f32_array(const uint16_t* src, float* dst, size_t n) {
  for (size_t i = 0; i < n; i++) dst[i] = or_f16_to_f32(src[i]);
}
void or_f32_to_bf16_array(const float* src, uint16_t* dst, size_t n) {
  for (size_t i = 0; i < n; i++) dst[i] = or_f32_to_bf16(src[i]);
}
void or_bf16_to_f32_array(const uint16_t* src, float* dst, size_t n) {
  for (size_t i = 0; i < n; i++) dst[i] = or_bf16_to_f32(src[i]);
}

/* ------------------------------------------------------------------ ops ---- */

/* src/core/ops.js:66-78. max over f32, exp in f64 stored to f32, the sum of
 * the unrounded f64 exps, then x = f32(x * (1/sum)). */
void or_softmax_inplace(float* x, int n) {
  float max = -INFINITY;
  for (int i = 0; i < n; i++) if (x[i] > max) max = x[i];
  double sum = 0.0;
  for (int i = 0; i < n; i++) {
    double e = exp((double)x[i] - (double)max);
    x[i] = (float)e;
    sum += e;
  }
  double inv = 1.0 / sum;
  for (int i = 0; i < n; i++) x[i] = (float)((double)x[i] * inv);
}

/* src/core/ops.js:99-104 -- inv_freq[j] = theta^(-2j/headDim). */
void or_rope_frequencies(int head_dim, double theta, double* inv_freq) {
  int half = head_dim >> 1;
  for (int j = 0; j < half; j++) inv_freq[j] = pow(theta, (double)(-2 * j) / (double)head_dim);
}

/* src/core/ops.js:123-136 -- f32 tables computed in f64. */
void or_rope_tables(int head_dim, double theta, int positions, float* cos_out, float* sin_out) {
  int half = head_dim >> 1;
  double* inv = (double*)malloc(sizeof(double) * (size_t)(half > 0 ? half : 1));
  or_rope_frequencies(head_dim, theta, inv);
  for (int p = 0; p < positions; p++) {
    for (int j = 0; j < half; j++) {
      double angle = (double)p * inv[j];
      cos_out[(size_t)p * half + j] = (float)cos(angle);
      sin_out[(size_t)p * half + j] = (float)sin(angle);
    }
  }
  free(inv);
}

/* The f64 angles of ops.js:147-152 (angle = position * invFreq[j]) tabulated
 * without the f32 rounding of ropeTables: exactly the cos/sin ropeInPlace
 * evaluates for that position. */
void or_rope_tables_f64(int head_dim, double theta, int positions, double* cos_out, double* sin_out) {
  int half = head_dim >> 1;
  double* inv = (double*)malloc(sizeof(double) * (size_t)(half > 0 ? half : 1));
  or_rope_frequencies(head_dim, theta, inv);
  for (int p = 0; p < positions; p++) {
    for (int j = 0; j < half; j++) {
      double angle = (double)p * inv[j];
      cos_out[(size_t)p * half + j] = cos(angle);
      sin_out[(size_t)p * half + j] = sin(angle);
    }
  }
  free(inv);
}

/* src/core/ops.js:147-158 -- half-split rotation in f64, stored to f32. */
void or_rope_inplace(float* vec, int offset, int head_dim, int position, const double* inv_freq) {
  int half = head_dim >> 1;
  for (int j = 0; j < half; j++) {
    double angle = (double)position * inv_freq[j];
    double c = cos(angle);
    double s = sin(angle);
    double lo = vec[offset + j];
    double hi = vec[offset + j + half];
    vec[offset + j] = (float)(lo * c - hi * s);
    vec[offset + j + half] = (float)(hi * c + lo * s);
  }
}

/* ------------------------------------------------------------ attention ---- */

/* src/core/attention.js:74-76 -- the blocked mapping. */
int or_kv_head_for(int query_head, int num_heads, int num_kv_heads) {
  return query_head / (num_heads / num_kv_heads);
}

/* src/core/attention.js:32-66. f64 dot of f32 operands, score stored to f32,
 * softmax (ops.js:66-78), then out = f32(out + f64(p * v)) in key order. */
void or_grouped_attention(const float* q, const float* keys, const float* values,
                          float* out, float* scores, int seq, int past,
                          int num_heads, int num_kv_heads, int head_dim) {
  int group = num_heads / num_kv_heads;
  int q_dim = num_heads * head_dim;
  int kv_dim = num_kv_heads * head_dim;
  double scale = 1.0 / sqrt((double)head_dim);
  memset(out, 0, sizeof(float) * (size_t)seq * q_dim);
  for (int h = 0; h < num_heads; h++) {
    int kv_base = (h / group) * head_dim;
    for (int t = 0; t < seq; t++) {
      int q_base = t * q_dim + h * head_dim;
      int up_to = past + t;
      for (int s = 0; s <= up_to; s++) {
        size_t k_base = (size_t)s * kv_dim + kv_base;
        double dot = 0.0;
        for (int i = 0; i < head_dim; i++) dot += (double)q[q_base + i] * (double)keys[k_base + i];
        scores[s] = (float)(dot * scale);
      }
      or_softmax_inplace(scores, up_to + 1);
      int out_base = t * q_dim + h * head_dim;
      for (int s = 0; s <= up_to; s++) {
        double w = scores[s];
        size_t v_base = (size_t)s * kv_dim + kv_base;
        for (int i = 0; i < head_dim; i++) {
          out[out_base + i] = (float)((double)out[out_base + i] + w * (double)values[v_base + i]);
        }
      }
    }
  }
}

/* test/attention.test.js:15-58 -- repeat each KV head groupSize times, then
 * plain multi-head attention. */
void or_expanded_attention(const float* q, const float* keys, const float* values,
                           float* out, int seq, int past,
                           int num_heads, int num_kv_heads, int head_dim) {
  int group = num_heads / num_kv_heads;
  int q_dim = num_heads * head_dim;
  int kv_dim = num_kv_heads * head_dim;
  int total = past + seq;
  float* wk = (float*)malloc(sizeof(float) * (size_t)total * q_dim);
  float* wv = (float*)malloc(sizeof(float) * (size_t)total * q_dim);
  float* scores = (float*)malloc(sizeof(float) * (size_t)(total > 0 ? total : 1));
  for (int s = 0; s < total; s++) {
    for (int h = 0; h < num_heads; h++) {
      size_t from = (size_t)s * kv_dim + (size_t)(h / group) * head_dim;
      size_t to = (size_t)s * q_dim + (size_t)h * head_dim;
      for (int i = 0; i < head_dim; i++) { wk[to + i] = keys[from + i]; wv[to + i] = values[from + i]; }
    }
  }
  memset(out, 0, sizeof(float) * (size_t)seq * q_dim);
  double scale = 1.0 / sqrt((double)head_dim);
  for (int h = 0; h < num_heads; h++) {
    for (int t = 0; t < seq; t++) {
      int up_to = past + t;
      int q_base = t * q_dim + h * head_dim;
      for (int s = 0; s <= up_to; s++) {
        double dot = 0.0;
        size_t k_base = (size_t)s * q_dim + (size_t)h * head_dim;
        for (int i = 0; i < head_dim; i++) dot += (double)q[q_base + i] * (double)wk[k_base + i];
        scores[s] = (float)(dot * scale);
      }
      or_softmax_inplace(scores, up_to + 1);
      int out_base = t * q_dim + h * head_dim;
      for (int s = 0; s <= up_to; s++) {
        size_t v_base = (size_t)s * q_dim + (size_t)h * head_dim;
        for (int i = 0; i < head_dim; i++) {
          out[out_base + i] = (float)((double)out[out_base + i] + (double)scores[s] * (double)wv[v_base + i]);
        }
      }
    }
  }
  free(wk); free(wv); free(scores);
}

/* ------------------------------------------------------------- KV cache ---- */

struct or_kvcache {
  int num_layers, kv_dim, capacity, length;
  float** keys;
  float** values;
};

/* src/cpu/cache.js:23-35 */
or_kvcache* or_kvcache_new(int num_layers, int kv_dim, int capacity, char* err, size_t errlen) {
  if (capacity < 1) {
    if (err) snprintf(err, errlen, "cache capacity must be a positive integer, got %d", capacity);
    return NULL;
  }
  or_kvcache* c = (or_kvcache*)calloc(1, sizeof(or_kvcache));
  c->num_layers = num_layers;
  c->kv_dim = kv_dim;
  c->capacity = capacity;
  c->keys = (float**)calloc((size_t)num_layers, sizeof(float*));
  c->values = (float**)calloc((size_t)num_layers, sizeof(float*));
  for (int l = 0; l < num_layers; l++) {
    c->keys[l] = (float*)calloc((size_t)capacity * kv_dim, sizeof(float));
    c->values[l] = (float*)calloc((size_t)capacity * kv_dim, sizeof(float));
  }
  return c;
}

void or_kvcache_free(or_kvcache* c) {
  if (!c) return;
  for (int l = 0; l < c->num_layers; l++) { free(c->keys[l]); free(c->values[l]); }
  free(c->keys); free(c->values); free(c);
}

int or_kvcache_length(const or_kvcache* c) { return c->length; }
int or_kvcache_capacity(const or_kvcache* c) { return c->capacity; }

/* src/cpu/cache.js:41-43 */
size_t or_kvcache_byte_length(const or_kvcache* c) {
  return (size_t)c->num_layers * c->capacity * c->kv_dim * 4 * 2;
}

/* src/cpu/cache.js:52-60 */
int or_kvcache_allocate(or_kvcache* c, int count, char* err, size_t errlen) {
  if (c->length + count > c->capacity) {
    if (err) snprintf(err, errlen, "cache holds %d of %d positions; cannot add %d more",
                      c->length, c->capacity, count);
    return -1;
  }
  return c->length;
}

/* src/cpu/cache.js:63-67 */
void or_kvcache_write_at(or_kvcache* c, int layer, int at, const float* keys,
                         const float* values, int count) {
  memcpy(c->keys[layer] + (size_t)at * c->kv_dim, keys, sizeof(float) * (size_t)count * c->kv_dim);
  memcpy(c->values[layer] + (size_t)at * c->kv_dim, values, sizeof(float) * (size_t)count * c->kv_dim);
}

/* src/cpu/cache.js:75-81 -- views; n is the caller's horizon (may exceed length). */
const float* or_kvcache_keys_up_to(const or_kvcache* c, int layer, int n) { (void)n; return c->keys[layer]; }
const float* or_kvcache_values_up_to(const or_kvcache* c, int layer, int n) { (void)n; return c->values[layer]; }

/* src/cpu/cache.js:84-86 */
void or_kvcache_commit(or_kvcache* c, int count) { c->length += count; }

/* src/cpu/cache.js:97-115 -- [kvHeads, length, headDim]. */
void or_kvcache_present(const or_kvcache* c, int layer, int num_kv_heads, int head_dim,
                        float* key_out, float* value_out) {
  int n = c->length;
  const float* k = c->keys[layer];
  const float* v = c->values[layer];
  for (int h = 0; h < num_kv_heads; h++) {
    for (int t = 0; t < n; t++) {
      size_t from = (size_t)t * c->kv_dim + (size_t)h * head_dim;
      size_t to = ((size_t)h * n + t) * head_dim;
      for (int i = 0; i < head_dim; i++) { key_out[to + i] = k[from + i]; value_out[to + i] = v[from + i]; }
    }
  }
}

/* src/cpu/cache.js:118 */
void or_kvcache_reset(or_kvcache* c) { c->length = 0; }

/* src/cpu/model.js:103-123 -- rope at absolute position past+t, append, attend. */
void or_layer_attention(or_kvcache* c, int layer, float* q, float* k, const float* v,
                        float* out, int seq, int num_heads, int num_kv_heads, int head_dim,
                        const double* inv_freq) {
  int past = c->length;
  int q_dim = num_heads * head_dim;
  int kv_dim = num_kv_heads * head_dim;
  for (int t = 0; t < seq; t++) {
    int position = past + t;
    for (int h = 0; h < num_heads; h++) or_rope_inplace(q, t * q_dim + h * head_dim, head_dim, position, inv_freq);
    for (int h = 0; h < num_kv_heads; h++) or_rope_inplace(k, t * kv_dim + h * head_dim, head_dim, position, inv_freq);
  }
  or_kvcache_write_at(c, layer, past, k, v, seq);
  float* scores = (float*)malloc(sizeof(float) * (size_t)(past + seq));
  or_grouped_attention(q, c->keys[layer], c->values[layer], out, scores, seq, past,
                       num_heads, num_kv_heads, head_dim);
  free(scores);
}

/* ------------------------------------------------------- decode helpers ---- */

/* attention.js:42-63 for seq=1, past=len, reading a head-major cache. */
void or_decode_head_major(const float* q, const float* kcache, const float* vcache,
                          int cap, int len, int num_heads, int num_kv_heads,
                          int head_dim, float* out) {
  int group = num_heads / num_kv_heads;
  double scale = 1.0 / sqrt((double)head_dim);
  float* scores = (float*)malloc(sizeof(float) * (size_t)(len + 1));
  for (int h = 0; h < num_heads; h++) {
    int g = h / group;
    const float* kh = kcache + (size_t)g * cap * head_dim;
    const float* vh = vcache + (size_t)g * cap * head_dim;
    const float* qh = q + (size_t)h * head_dim;
    for (int s = 0; s <= len; s++) {
      double dot = 0.0;
      for (int i = 0; i < head_dim; i++) dot += (double)qh[i] * (double)kh[(size_t)s * head_dim + i];
      scores[s] = (float)(dot * scale);
    }
    or_softmax_inplace(scores, len + 1);
    float* oh = out + (size_t)h * head_dim;
    for (int i = 0; i < head_dim; i++) oh[i] = 0.0f;
    for (int s = 0; s <= len; s++) {
      double w = scores[s];
      for (int i = 0; i < head_dim; i++) oh[i] = (float)((double)oh[i] + w * (double)vh[(size_t)s * head_dim + i]);
    }
  }
  free(scores);
}

/* One chunk of the split-KV decomposition of attention.js:49-62: the softmax of
 * ops.js:66-78 with its normalisation deferred. Natural-log units. */
void or_decode_partial(const float* qh, const float* kh, const float* vh,
                       int p0, int p1, int head_dim, float* m, float* l, float* o) {
  double scale = 1.0 / sqrt((double)head_dim);
  int n = p1 - p0;
  float* scores = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
  float mx = -INFINITY;
  for (int s = 0; s < n; s++) {
    double dot = 0.0;
    for (int i = 0; i < head_dim; i++) dot += (double)qh[i] * (double)kh[(size_t)(p0 + s) * head_dim + i];
    scores[s] = (float)(dot * scale);
    if (scores[s] > mx) mx = scores[s];
  }
  double sum = 0.0;
  double* acc = (double*)calloc((size_t)head_dim, sizeof(double));
  for (int s = 0; s < n; s++) {
    double e = exp((double)scores[s] - (double)mx);
    sum += e;
    for (int i = 0; i < head_dim; i++) acc[i] += e * (double)vh[(size_t)(p0 + s) * head_dim + i];
  }
  *m = mx;
  *l = (float)sum;
  for (int i = 0; i < head_dim; i++) o[i] = (float)acc[i];
  free(acc);
  free(scores);
}

/* m* = max m_g; l* = sum e^(m_g-m*) l_g; out = sum e^(m_g-m*) o_g / l*, in
 * ascending g so every caller gets the same bits. Empty partials (l == 0)
 * contribute nothing. */
void or_lse_combine(const float* m, const float* l, const float* o, int g,
                    int head_dim, float* out) {
  double mx = -INFINITY;
  for (int i = 0; i < g; i++) if (l[i] > 0.0f && m[i] > mx) mx = m[i];
  double lsum = 0.0;
  double* acc = (double*)calloc((size_t)head_dim, sizeof(double));
  for (int i = 0; i < g; i++) {
    if (!(l[i] > 0.0f)) continue;
    double w = exp((double)m[i] - mx);
    lsum += w * (double)l[i];
    for (int d = 0; d < head_dim; d++) acc[d] += w * (double)o[(size_t)i * head_dim + d];
  }
  for (int d = 0; d < head_dim; d++) out[d] = (float)(acc[d] / lsum);
  free(acc);
}

/* ----------------------------------------------------------- generators ---- */

/* test/attention.test.js:60-69 */
void or_random_array(float* out, size_t n, uint32_t seed) {
  uint32_t state = seed;
  for (size_t i = 0; i < n; i++) {
    state = state * 1664525u + 1013904223u;
    out[i] = (float)(((double)state / 4294967295.0) * 2.0 - 1.0);
  }
}

static inline uint64_t splitmix64(uint64_t* s) {
  uint64_t z = (*s += 0x9e3779b97f4a7c15ull);
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

/* splitmix64 uniforms (53-bit) into Box-Muller pairs. */
void or_normal_array(float* out, size_t n, uint64_t seed) {
  uint64_t s = seed;
  const double two_pi = 6.283185307179586;
  for (size_t i = 0; i < n; i += 2) {
    double u1 = ((double)(splitmix64(&s) >> 11) + 1.0) * (1.0 / 9007199254740992.0); /* (0,1] */
    double u2 = (double)(splitmix64(&s) >> 11) * (1.0 / 9007199254740992.0);         /* [0,1) */
    double r = sqrt(-2.0 * log(u1));
    out[i] = (float)(r * cos(two_pi * u2));
    if (i + 1 < n) out[i + 1] = (float)(r * sin(two_pi * u2));
  }
}

/* ------------------------------------------------- CPU baseline (batched) -- */

static float g_f16_table[65536];
static int g_f16_table_ready = 0;

static void f16_table_init(void) {
  if (g_f16_table_ready) return;
  for (uint32_t h = 0; h < 65536; h++) g_f16_table[h] = or_f16_to_f32((uint16_t)h);
  g_f16_table_ready = 1;
}

int or_batched_decode_f16(const float* q, size_t q_stride, const uint16_t* kcache,
                          const uint16_t* vcache, size_t seq_stride, const int32_t* len,
                          int batch, int cap, int num_heads, int num_kv_heads, int head_dim,
                          float* out, size_t out_stride, int threads) {
  f16_table_init();
  int used = 1;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_num_procs();
  used = threads;
#else
  (void)threads;
#endif
  int group = num_heads / num_kv_heads;
  double scale = 1.0 / sqrt((double)head_dim);
  long pairs = (long)batch * num_heads;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
#endif
  for (long bh = 0; bh < pairs; bh++) {
    int b = (int)(bh / num_heads);
    int h = (int)(bh % num_heads);
    int g = h / group;
    int n = len[b] + 1;
    const uint16_t* kh = kcache + (size_t)b * seq_stride + (size_t)g * cap * head_dim;
    const uint16_t* vh = vcache + (size_t)b * seq_stride + (size_t)g * cap * head_dim;
    const float* qh = q + (size_t)b * q_stride + (size_t)h * head_dim;
    float* scores = (float*)malloc(sizeof(float) * (size_t)n);
    for (int s = 0; s < n; s++) {
      double dot = 0.0;
      const uint16_t* kr = kh + (size_t)s * head_dim;
      for (int i = 0; i < head_dim; i++) dot += (double)qh[i] * (double)g_f16_table[kr[i]];
      scores[s] = (float)(dot * scale);
    }
    or_softmax_inplace(scores, n);
    float* oh = out + (size_t)b * out_stride + (size_t)h * head_dim;
    for (int i = 0; i < head_dim; i++) oh[i] = 0.0f;
    for (int s = 0; s < n; s++) {
      double w = scores[s];
      const uint16_t* vr = vh + (size_t)s * head_dim;
      for (int i = 0; i < head_dim; i++) oh[i] = (float)((double)oh[i] + w * (double)g_f16_table[vr[i]]);
    }
    free(scores);
  }
  return used;
}

/* ------------------------------------------------------------------ projections */

/* src/core/quantize.js:25-27: round half away from zero (C's round). */
void or_quantize_int8_per_channel(const float* w, int rows, int cols, int8_t* codes, float* scales) {
  for (int r = 0; r < rows; r++) {
    const float* row = w + (size_t)r * cols;
    double peak = 0.0;
    for (int c = 0; c < cols; c++) {
      const double m = fabs((double)row[c]);
      if (m > peak) peak = m;
    }
    const double scale = peak / 127.0;            /* a JS number: f64 */
    scales[r] = (float)scale;                     /* Float32Array store */
    int8_t* out = codes + (size_t)r * cols;
    if (scale == 0.0) {
      memset(out, 0, (size_t)cols);
      continue;
    }
    const double inverse = 1.0 / scale;
    for (int c = 0; c < cols; c++) {
      double level = round((double)row[c] * inverse);
      if (level > 127.0) level = 127.0;
      if (level < -127.0) level = -127.0;
      out[c] = (int8_t)level;
    }
  }
}

void or_dequantize_int8_per_channel(const int8_t* codes, const float* scales, int rows, int cols, float* out) {
  for (int r = 0; r < rows; r++) {
    const double s = (double)scales[r];
    for (int c = 0; c < cols; c++) out[(size_t)r * cols + c] = (float)((double)codes[(size_t)r * cols + c] * s);
  }
}

void or_matvec(const float* w, const float* x, int rows, int cols, const float* bias, float* out) {
  for (int r = 0; r < rows; r++) {
    double acc = bias ? (double)bias[r] : 0.0;
    const float* row = w + (size_t)r * cols;
    for (int c = 0; c < cols; c++) acc += (double)row[c] * (double)x[c];
    out[r] = (float)acc;
  }
}

/* ------------------------------------------------ the decoder around attention -- */

/* src/core/ops.js:17-24: f64 sum of squares, scale = 1/sqrt(ss/n + eps), out = x*scale*w. */
void or_rmsnorm(const float* x, const float* weight, double eps, int n, float* out) {
  double sum_squares = 0.0;
  for (int i = 0; i < n; i++) sum_squares += (double)x[i] * (double)x[i];
  const double scale = 1.0 / sqrt(sum_squares / n + eps);
  for (int i = 0; i < n; i++) out[i] = (float)((double)x[i] * scale * (double)weight[i]);
}

/* src/core/ops.js:81-83 */
double or_silu(double x) { return x / (1.0 + exp(-x)); }

/* src/core/ops.js:88-91 */
void or_swiglu_inplace(float* gate, const float* up, int n) {
  for (int i = 0; i < n; i++) gate[i] = (float)(or_silu((double)gate[i]) * (double)up[i]);
}

/* src/cpu/model.js:181-183: the first index of the largest value. */
int or_argmax(const float* logits, int n) {
  int best = 0;
  for (int i = 1; i < n; i++)
    if (logits[i] > logits[best]) best = i;
  return best;
}

/* matVec (ops.js:33-41) over an int8 matrix widened per element exactly as
 * or_dequantize_int8_per_channel does (quantize.js:60-67), rows split over
 * `threads` OpenMP threads (each row's sum is the same either way). */
static void matvec_int8(const int8_t* codes, const float* scales, const float* x, int rows, int cols,
                        const float* bias, float* out, int threads) {
#pragma omp parallel for schedule(static) num_threads(threads) if (threads > 1)
  for (int r = 0; r < rows; r++) {
    const double s = (double)scales[r];
    const int8_t* row = codes + (size_t)r * cols;
    double acc = bias ? (double)bias[r] : 0.0;
    for (int c = 0; c < cols; c++) acc += (double)(float)((double)row[c] * s) * (double)x[c];
    out[r] = (float)acc;
  }
}

typedef struct {
  const float *in_norm, *post_norm, *qkv_scales, *qkv_bias, *o_scales, *gate_scales, *up_scales, *down_scales;
  const int8_t *qkv, *o, *gate, *up, *down;
} or_layer;

struct or_model {
  int hidden, inter, layers, heads, kv_heads, vocab, head_dim, threads;
  double eps;
  double* inv_freq;
  const int8_t* emb;
  const float* emb_scales;
  const float* final_norm;
  or_layer* w;
  or_kvcache* cache;
};

or_model* or_model_new(int hidden, int inter, int layers, int heads, int kv_heads, int vocab, double theta,
                       double eps, int capacity, int threads) {
  or_model* m = (or_model*)calloc(1, sizeof(or_model));
  m->hidden = hidden;
  m->inter = inter;
  m->layers = layers;
  m->heads = heads;
  m->kv_heads = kv_heads;
  m->vocab = vocab;
  m->head_dim = hidden / heads;
  m->eps = eps;
  m->threads = threads > 0 ? threads : 1;
  m->inv_freq = (double*)malloc(sizeof(double) * (size_t)(m->head_dim / 2));
  or_rope_frequencies(m->head_dim, theta, m->inv_freq);
  m->w = (or_layer*)calloc((size_t)layers, sizeof(or_layer));
  m->cache = or_kvcache_new(layers, kv_heads * m->head_dim, capacity, NULL, 0);
  return m;
}

void or_model_free(or_model* m) {
  if (!m) return;
  or_kvcache_free(m->cache);
  free(m->inv_freq);
  free(m->w);
  free(m);
}

void or_model_set_layer(or_model* m, int layer, const float* in_norm, const float* post_norm, const int8_t* qkv,
                        const float* qkv_scales, const float* qkv_bias, const int8_t* o, const float* o_scales,
                        const int8_t* gate, const float* gate_scales, const int8_t* up, const float* up_scales,
                        const int8_t* down, const float* down_scales) {
  or_layer* w = &m->w[layer];
  w->in_norm = in_norm;
  w->post_norm = post_norm;
  w->qkv = qkv;
  w->qkv_scales = qkv_scales;
  w->qkv_bias = qkv_bias;
  w->o = o;
  w->o_scales = o_scales;
  w->gate = gate;
  w->gate_scales = gate_scales;
  w->up = up;
  w->up_scales = up_scales;
  w->down = down;
  w->down_scales = down_scales;
}

void or_model_set_embedding(or_model* m, const int8_t* codes, const float* scales, const float* final_norm) {
  m->emb = codes;
  m->emb_scales = scales;
  m->final_norm = final_norm;
}

int or_model_length(const or_model* m) { return or_kvcache_length(m->cache); }
void or_model_reset(or_model* m) { or_kvcache_reset(m->cache); }

void or_model_present(const or_model* m, int layer, float* key_out, float* value_out) {
  or_kvcache_present(m->cache, layer, m->kv_heads, m->head_dim, key_out, value_out);
}

static float round_f16(float x) { return or_f16_to_f32(or_f32_to_f16(x)); }

/* ReferenceModel.forward (src/cpu/model.js:55-161) over the int8 weights,
 * with the device path's dtype boundaries restated: q/k/v are rounded to f16
 * after their projection (the attention kernels take 16-bit inputs) and the
 * cache keeps RoPE(k) and v rounded to f16 (the f16 cache). Everything else is
 * the reference's f32 storage with f64 reductions. Returns the greedy pick of
 * the last position's logits ([vocab], may be NULL) or -1 with err filled. */
int or_model_forward(or_model* m, const int32_t* tokens, int seq, float* logits_out, char* err, size_t errlen) {
  const int d = m->hidden, kv_dim = m->kv_heads * m->head_dim, ffn = m->inter;
  if (seq < 1) {
    if (err) snprintf(err, errlen, "forward: need at least one token");
    return -1;
  }
  for (int t = 0; t < seq; t++) {
    if (tokens[t] < 0 || tokens[t] >= m->vocab) {
      if (err) snprintf(err, errlen, "token %d at position %d is outside the vocabulary", tokens[t], t);
      return -1;
    }
  }
  const int past = or_kvcache_allocate(m->cache, seq, err, errlen);
  if (past < 0) return -1;
  const int total = past + seq;
  float* x = (float*)malloc(sizeof(float) * (size_t)seq * d);
  float* normed = (float*)malloc(sizeof(float) * (size_t)d);
  float* qkv = (float*)malloc(sizeof(float) * (size_t)(d + 2 * kv_dim));
  float* q = (float*)malloc(sizeof(float) * (size_t)seq * d);
  float* k = (float*)malloc(sizeof(float) * (size_t)seq * kv_dim);
  float* v = (float*)malloc(sizeof(float) * (size_t)seq * kv_dim);
  float* att = (float*)malloc(sizeof(float) * (size_t)seq * d);
  float* scores = (float*)malloc(sizeof(float) * (size_t)total);
  float* gate = (float*)malloc(sizeof(float) * (size_t)ffn);
  float* up = (float*)malloc(sizeof(float) * (size_t)ffn);
  float* projected = (float*)malloc(sizeof(float) * (size_t)d);
  float* logits = (float*)malloc(sizeof(float) * (size_t)m->vocab);

  /* #embed (model.js:195-210) of the int8 table */
  for (int t = 0; t < seq; t++) {
    const double s = (double)m->emb_scales[tokens[t]];
    const int8_t* row = m->emb + (size_t)tokens[t] * d;
    for (int i = 0; i < d; i++) x[(size_t)t * d + i] = (float)((double)row[i] * s);
  }
  for (int layer = 0; layer < m->layers; layer++) {
    const or_layer* w = &m->w[layer];
    for (int t = 0; t < seq; t++) {
      or_rmsnorm(x + (size_t)t * d, w->in_norm, m->eps, d, normed);
      matvec_int8(w->qkv, w->qkv_scales, normed, d + 2 * kv_dim, d, w->qkv_bias, qkv, m->threads);
      for (int i = 0; i < d; i++) q[(size_t)t * d + i] = round_f16(qkv[i]);
      for (int i = 0; i < kv_dim; i++) {
        k[(size_t)t * kv_dim + i] = round_f16(qkv[d + i]);
        v[(size_t)t * kv_dim + i] = round_f16(qkv[d + kv_dim + i]);
      }
      const int position = past + t;
      for (int h = 0; h < m->heads; h++) or_rope_inplace(q, t * d + h * m->head_dim, m->head_dim, position, m->inv_freq);
      for (int h = 0; h < m->kv_heads; h++) {
        or_rope_inplace(k, t * kv_dim + h * m->head_dim, m->head_dim, position, m->inv_freq);
      }
      for (int i = 0; i < kv_dim; i++) k[(size_t)t * kv_dim + i] = round_f16(k[(size_t)t * kv_dim + i]);
    }
    or_kvcache_write_at(m->cache, layer, past, k, v, seq);
    or_grouped_attention(q, or_kvcache_keys_up_to(m->cache, layer, total),
                         or_kvcache_values_up_to(m->cache, layer, total), att, scores, seq, past, m->heads,
                         m->kv_heads, m->head_dim);
    for (int t = 0; t < seq; t++) {
      matvec_int8(w->o, w->o_scales, att + (size_t)t * d, d, d, NULL, projected, m->threads);
      for (int i = 0; i < d; i++) x[(size_t)t * d + i] += projected[i];
    }
    for (int t = 0; t < seq; t++) {
      float* row = x + (size_t)t * d;
      or_rmsnorm(row, w->post_norm, m->eps, d, normed);
      matvec_int8(w->gate, w->gate_scales, normed, ffn, d, NULL, gate, m->threads);
      matvec_int8(w->up, w->up_scales, normed, ffn, d, NULL, up, m->threads);
      or_swiglu_inplace(gate, up, ffn);
      matvec_int8(w->down, w->down_scales, gate, d, ffn, NULL, projected, m->threads);
      for (int i = 0; i < d; i++) row[i] += projected[i];
    }
  }
  or_kvcache_commit(m->cache, seq);
  or_rmsnorm(x + (size_t)(seq - 1) * d, m->final_norm, m->eps, d, normed);
  matvec_int8(m->emb, m->emb_scales, normed, m->vocab, d, NULL, logits, m->threads);
  const int best = or_argmax(logits, m->vocab);
  if (logits_out) memcpy(logits_out, logits, sizeof(float) * (size_t)m->vocab);
  free(x);
  free(normed);
  free(qkv);
  free(q);
  free(k);
  free(v);
  free(att);
  free(scores);
  free(gate);
  free(up);
  free(projected);
  free(logits);
  return best;
}
