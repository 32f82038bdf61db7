/*
 * b2a_napi.c -- Node-API addon over libb2a.so: the binding a maintainer of
 * abho7/llm-inference-webgpu would add so its model loop calls the B200 path
 * through the operator surface it already uses.
 *
 * Runtime-unverified: there is no Node.js on the machines this repository is
 * built and tested on, and no node_api.h. Without B2A_HAVE_NODE_API_H the
 * N-API functions used below are declared here by hand, exactly as the stable
 * C ABI (N-API version 1+) defines them; the file is compile-checked that way
 * with `gcc -fsyntax-only -Wall -Wextra -Werror -I include addon/b2a_napi.c`
 * (tests/test_abi_cpu.py). binding.gyp beside this file builds it with
 * node-gyp against Node's own node_api.h and links libb2a.so.
 *
 * Bound surface (reference file:line it replaces):
 *   groupedAttention(q, keys, values, out, scores, shape)  src/core/attention.js:32-66
 *   kvHeadFor(h, numHeads, numKVHeads)                     src/core/attention.js:74-76
 *   ropeFrequencies(headDim, theta)                        src/core/ops.js:99-104
 *   ropeTables(headDim, theta, positions)                  src/core/ops.js:123-136
 *   new KVCache(config, capacity) and its methods          src/cpu/cache.js:18-119
 *     allocate / writeAt / keysUpTo / valuesUpTo / present / commit / length / reset
 *   attentionDecode / attentionPrefill (the GPU loop's rope-q, rope-k, append and
 *     ATTENTION dispatches fused into one call)            src/gpu/model.js:323-346
 * Errors: B2A_ERANGE becomes the reference's RangeError with the same message
 * text (src/cpu/cache.js:24-26, 53-58); everything else an Error whose code is
 * the status name. The addon owns one context (the reference's GpuContext,
 * src/gpu/device.js:21), created when the module loads.
 */
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "b2a.h"

#ifdef B2A_HAVE_NODE_API_H
#include <node_api.h>
#else
/* ---- the N-API declarations this file uses (stable C ABI) ----------------- */
typedef struct napi_env__* napi_env;
typedef struct napi_value__* napi_value;
typedef struct napi_callback_info__* napi_callback_info;
typedef enum { napi_ok = 0 } napi_status;
typedef enum {
  napi_int8_array, napi_uint8_array, napi_uint8_clamped_array, napi_int16_array, napi_uint16_array,
  napi_int32_array, napi_uint32_array, napi_float32_array, napi_float64_array, napi_bigint64_array,
  napi_biguint64_array
} napi_typedarray_type;
typedef napi_value (*napi_callback)(napi_env env, napi_callback_info info);
typedef void (*napi_finalize)(napi_env env, void* finalize_data, void* finalize_hint);
#define NAPI_AUTO_LENGTH SIZE_MAX

napi_status napi_get_cb_info(napi_env env, napi_callback_info cbinfo, size_t* argc, napi_value* argv,
                             napi_value* this_arg, void** data);
napi_status napi_get_typedarray_info(napi_env env, napi_value typedarray, napi_typedarray_type* type,
                                     size_t* length, void** data, napi_value* arraybuffer, size_t* byte_offset);
napi_status napi_create_arraybuffer(napi_env env, size_t byte_length, void** data, napi_value* result);
napi_status napi_create_typedarray(napi_env env, napi_typedarray_type type, size_t length, napi_value arraybuffer,
                                   size_t byte_offset, napi_value* result);
napi_status napi_get_named_property(napi_env env, napi_value object, const char* utf8name, napi_value* result);
napi_status napi_set_named_property(napi_env env, napi_value object, const char* utf8name, napi_value value);
napi_status napi_get_value_int32(napi_env env, napi_value value, int32_t* result);
napi_status napi_get_value_double(napi_env env, napi_value value, double* result);
napi_status napi_create_int32(napi_env env, int32_t value, napi_value* result);
napi_status napi_create_double(napi_env env, double value, napi_value* result);
napi_status napi_create_object(napi_env env, napi_value* result);
napi_status napi_get_undefined(napi_env env, napi_value* result);
napi_status napi_create_external(napi_env env, void* data, napi_finalize finalize_cb, void* finalize_hint,
                                 napi_value* result);
napi_status napi_get_value_external(napi_env env, napi_value value, void** result);
napi_status napi_create_function(napi_env env, const char* utf8name, size_t length, napi_callback cb, void* data,
                                 napi_value* result);
napi_status napi_throw_error(napi_env env, const char* code, const char* msg);
napi_status napi_throw_type_error(napi_env env, const char* code, const char* msg);
napi_status napi_throw_range_error(napi_env env, const char* code, const char* msg);
/* ---- end of the N-API declarations ---------------------------------------- */
#endif

static b2a_ctx* g_ctx;   /* one context per process, like the reference's GpuContext */

static napi_value throw_status(napi_env env, b2a_status s) {
  if (s == B2A_ERANGE) napi_throw_range_error(env, NULL, b2a_last_error());
  else napi_throw_error(env, b2a_status_name(s), b2a_last_error());
  return NULL;
}

static napi_value undefined(napi_env env) {
  napi_value u;
  napi_get_undefined(env, &u);
  return u;
}

/* Arguments: fails (with a pending TypeError) unless argv[i] is a typed array of `want`. */
static int arg_typed(napi_env env, napi_value v, napi_typedarray_type want, void** data, size_t* length) {
  napi_typedarray_type t;
  napi_value ab;
  size_t off;
  if (napi_get_typedarray_info(env, v, &t, length, data, &ab, &off) != napi_ok || t != want) {
    napi_throw_type_error(env, NULL, want == napi_float32_array ? "expected a Float32Array" : "expected a typed array");
    return 0;
  }
  return 1;
}

static int arg_int(napi_env env, napi_value v, int32_t* out) {
  if (napi_get_value_int32(env, v, out) != napi_ok) {
    napi_throw_type_error(env, NULL, "expected an integer");
    return 0;
  }
  return 1;
}

static int prop_int(napi_env env, napi_value obj, const char* name, int32_t* out) {
  napi_value x;
  return napi_get_named_property(env, obj, name, &x) == napi_ok && arg_int(env, x, out);
}

static napi_value make_f32(napi_env env, size_t n, float** data) {
  napi_value ab, arr;
  void* p = NULL;
  if (napi_create_arraybuffer(env, n * sizeof(float), &p, &ab) != napi_ok) return NULL;
  if (napi_create_typedarray(env, napi_float32_array, n, ab, 0, &arr) != napi_ok) return NULL;
  *data = (float*)p;
  return arr;
}

/* groupedAttention(q, keys, values, out, scores, {seq, past, numHeads, numKVHeads, headDim}) -> out
 * (src/core/attention.js:32-66; `scores` is accepted and unused: the kernel keeps its own). */
static napi_value GroupedAttention(napi_env env, napi_callback_info info) {
  size_t argc = 6;
  napi_value argv[6];
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  if (argc < 6) {
    napi_throw_type_error(env, NULL, "groupedAttention(q, keys, values, out, scores, shape)");
    return NULL;
  }
  void *q, *k, *v, *out;
  size_t n;
  int32_t seq, past, H, KVH, D;
  if (!arg_typed(env, argv[0], napi_float32_array, &q, &n) || !arg_typed(env, argv[1], napi_float32_array, &k, &n) ||
      !arg_typed(env, argv[2], napi_float32_array, &v, &n) || !arg_typed(env, argv[3], napi_float32_array, &out, &n) ||
      !prop_int(env, argv[5], "seq", &seq) || !prop_int(env, argv[5], "past", &past) ||
      !prop_int(env, argv[5], "numHeads", &H) || !prop_int(env, argv[5], "numKVHeads", &KVH) ||
      !prop_int(env, argv[5], "headDim", &D)) {
    return NULL;
  }
  b2a_status s = b2a_grouped_attention(g_ctx, q, k, v, out, NULL, seq, past, H, KVH, D, B2A_HOST);
  if (s != B2A_OK) return throw_status(env, s);
  return argv[3];
}

/* kvHeadFor(queryHead, numHeads, numKVHeads) (src/core/attention.js:74-76) */
static napi_value KvHeadFor(napi_env env, napi_callback_info info) {
  size_t argc = 3;
  napi_value argv[3], r;
  int32_t h, H, KVH;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  if (argc < 3 || !arg_int(env, argv[0], &h) || !arg_int(env, argv[1], &H) || !arg_int(env, argv[2], &KVH)) return NULL;
  napi_create_int32(env, b2a_kv_head_for(h, H, KVH), &r);
  return r;
}

/* ropeFrequencies(headDim, theta) -> Float64Array (src/core/ops.js:99-104) */
static napi_value RopeFrequencies(napi_env env, napi_callback_info info) {
  size_t argc = 2;
  napi_value argv[2], ab, arr;
  int32_t D;
  double theta;
  void* p = NULL;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  if (argc < 2 || !arg_int(env, argv[0], &D) || napi_get_value_double(env, argv[1], &theta) != napi_ok || D < 2) {
    napi_throw_type_error(env, NULL, "ropeFrequencies(headDim, theta)");
    return NULL;
  }
  napi_create_arraybuffer(env, (size_t)(D / 2) * sizeof(double), &p, &ab);
  napi_create_typedarray(env, napi_float64_array, (size_t)(D / 2), ab, 0, &arr);
  b2a_status s = b2a_rope_frequencies(D, theta, (double*)p);
  if (s != B2A_OK) return throw_status(env, s);
  return arr;
}

/* ropeTables(headDim, theta, positions) -> {cos, sin} Float32Arrays (src/core/ops.js:123-136) */
static napi_value RopeTables(napi_env env, napi_callback_info info) {
  size_t argc = 3;
  napi_value argv[3], obj, c, sn;
  int32_t D, P;
  double theta;
  float *cp, *sp;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  if (argc < 3 || !arg_int(env, argv[0], &D) || napi_get_value_double(env, argv[1], &theta) != napi_ok ||
      !arg_int(env, argv[2], &P) || D < 2 || P < 0) {
    napi_throw_type_error(env, NULL, "ropeTables(headDim, theta, positions)");
    return NULL;
  }
  c = make_f32(env, (size_t)P * (D / 2), &cp);
  sn = make_f32(env, (size_t)P * (D / 2), &sp);
  if (c == NULL || sn == NULL) return NULL;
  b2a_status s = b2a_rope_tables(D, theta, P, cp, sp);
  if (s != B2A_OK) return throw_status(env, s);
  napi_create_object(env, &obj);
  napi_set_named_property(env, obj, "cos", c);
  napi_set_named_property(env, obj, "sin", sn);
  return obj;
}

/* ---- KVCache (src/cpu/cache.js:18-119) over a device cache ------------------ */
typedef struct {
  b2a_kvcache* cache;
  int32_t layers, kv_heads, head_dim, capacity;
} Cache;

static void cache_finalize(napi_env env, void* data, void* hint) {
  (void)env;
  (void)hint;
  Cache* c = (Cache*)data;
  if (c->cache) b2a_kvcache_destroy(c->cache);
  free(c);
}

static Cache* arg_cache(napi_env env, napi_value v) {
  void* p = NULL;
  if (napi_get_value_external(env, v, &p) != napi_ok || p == NULL) {
    napi_throw_type_error(env, NULL, "expected a cache handle");
    return NULL;
  }
  return (Cache*)p;
}

/* kvCacheCreate({numLayers, numKVHeads, headDim}, capacity) -> handle.
 * capacity < 1: RangeError "cache capacity must be a positive integer, got N" (cache.js:24-26). */
static napi_value KvCacheCreate(napi_env env, napi_callback_info info) {
  size_t argc = 2;
  napi_value argv[2], r;
  Cache c = {0};
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  if (argc < 2 || !prop_int(env, argv[0], "numLayers", &c.layers) ||
      !prop_int(env, argv[0], "numKVHeads", &c.kv_heads) || !prop_int(env, argv[0], "headDim", &c.head_dim) ||
      !arg_int(env, argv[1], &c.capacity)) {
    return NULL;
  }
  b2a_status s = b2a_kvcache_create(g_ctx, c.layers, c.kv_heads, c.head_dim, c.capacity, 1, B2A_F32, &c.cache);
  if (s != B2A_OK) return throw_status(env, s);
  Cache* h = (Cache*)malloc(sizeof(Cache));
  if (h == NULL) {
    b2a_kvcache_destroy(c.cache);
    napi_throw_error(env, NULL, "out of host memory");
    return NULL;
  }
  *h = c;
  napi_create_external(env, h, cache_finalize, NULL, &r);
  return r;
}

/* allocate(count) -> first position; RangeError "cache holds L of C positions; cannot add K more" */
static napi_value KvCacheAllocate(napi_env env, napi_callback_info info) {
  size_t argc = 2;
  napi_value argv[2], r;
  int32_t count;
  int at = 0;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  Cache* c = argc >= 2 ? arg_cache(env, argv[0]) : NULL;
  if (c == NULL || !arg_int(env, argv[1], &count)) return NULL;
  b2a_status s = b2a_kvcache_allocate(c->cache, 0, count, &at);
  if (s != B2A_OK) return throw_status(env, s);
  napi_create_int32(env, at, &r);
  return r;
}

/* writeAt(layer, at, keys, values, count): rows [count][kvDim] f32 (cache.js:63-67) */
static napi_value KvCacheWriteAt(napi_env env, napi_callback_info info) {
  size_t argc = 6;
  napi_value argv[6];
  int32_t layer, at, count;
  void *k, *v;
  size_t n;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  Cache* c = argc >= 6 ? arg_cache(env, argv[0]) : NULL;
  if (c == NULL || !arg_int(env, argv[1], &layer) || !arg_int(env, argv[2], &at) ||
      !arg_typed(env, argv[3], napi_float32_array, &k, &n) || !arg_typed(env, argv[4], napi_float32_array, &v, &n) ||
      !arg_int(env, argv[5], &count)) {
    return NULL;
  }
  b2a_status s = b2a_kvcache_write_at(g_ctx, c->cache, layer, 0, at, k, v, B2A_F32, count, B2A_HOST);
  if (s != B2A_OK) return throw_status(env, s);
  return undefined(env);
}

/* keysUpTo / valuesUpTo (cache.js:75-82) as position-major [n][kvDim], and present()
 * (cache.js:97-115) as head-major [kvHeads][n][headDim]: which = 0 keys, 1 values, 2 present. */
static napi_value cache_read(napi_env env, napi_callback_info info, int which) {
  size_t argc = 3;
  napi_value argv[3];
  int32_t layer, n = 0;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  Cache* c = argc >= 2 ? arg_cache(env, argv[0]) : NULL;
  if (c == NULL || !arg_int(env, argv[1], &layer)) return NULL;
  if (which == 2) {
    b2a_status s = b2a_kvcache_length(c->cache, 0, &n);
    if (s != B2A_OK) return throw_status(env, s);
  } else if (argc < 3 || !arg_int(env, argv[2], &n)) {
    return NULL;
  }
  const size_t row = (size_t)c->kv_heads * c->head_dim, total = (size_t)n * row;
  float *hk = (float*)malloc(total * sizeof(float) + 1), *hv = (float*)malloc(total * sizeof(float) + 1);
  if (hk == NULL || hv == NULL) {
    free(hk);
    free(hv);
    napi_throw_error(env, NULL, "out of host memory");
    return NULL;
  }
  b2a_status s = b2a_kvcache_read(g_ctx, c->cache, layer, 0, n, hk, hv, B2A_HOST);   /* head-major */
  if (s != B2A_OK) {
    free(hk);
    free(hv);
    return throw_status(env, s);
  }
  napi_value result;
  float *dk, *dv;
  if (which == 2) {
    napi_value ka = make_f32(env, total, &dk), va = make_f32(env, total, &dv);
    memcpy(dk, hk, total * sizeof(float));
    memcpy(dv, hv, total * sizeof(float));
    napi_create_object(env, &result);
    napi_set_named_property(env, result, "key", ka);
    napi_set_named_property(env, result, "value", va);
  } else {
    /* back to the reference's position-major rows */
    const float* src = which == 0 ? hk : hv;
    result = make_f32(env, total, &dk);
    for (int32_t p = 0; p < n; p++)
      for (int32_t g = 0; g < c->kv_heads; g++)
        memcpy(dk + (size_t)p * row + (size_t)g * c->head_dim, src + ((size_t)g * n + p) * c->head_dim,
               (size_t)c->head_dim * sizeof(float));
  }
  free(hk);
  free(hv);
  return result;
}
static napi_value KvCacheKeysUpTo(napi_env env, napi_callback_info info) { return cache_read(env, info, 0); }
static napi_value KvCacheValuesUpTo(napi_env env, napi_callback_info info) { return cache_read(env, info, 1); }
static napi_value KvCachePresent(napi_env env, napi_callback_info info) { return cache_read(env, info, 2); }

/* commit(count) (cache.js:84-86) */
static napi_value KvCacheCommit(napi_env env, napi_callback_info info) {
  size_t argc = 2;
  napi_value argv[2];
  int32_t count;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  Cache* c = argc >= 2 ? arg_cache(env, argv[0]) : NULL;
  if (c == NULL || !arg_int(env, argv[1], &count)) return NULL;
  b2a_status s = b2a_kvcache_commit(c->cache, 0, count);
  if (s != B2A_OK) return throw_status(env, s);
  return undefined(env);
}

/* length (cache.js:38) */
static napi_value KvCacheLength(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1], r;
  int n = 0;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  Cache* c = argc >= 1 ? arg_cache(env, argv[0]) : NULL;
  if (c == NULL) return NULL;
  b2a_status s = b2a_kvcache_length(c->cache, 0, &n);
  if (s != B2A_OK) return throw_status(env, s);
  napi_create_int32(env, n, &r);
  return r;
}

/* reset() (cache.js:118) */
static napi_value KvCacheReset(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1];
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  Cache* c = argc >= 1 ? arg_cache(env, argv[0]) : NULL;
  if (c == NULL) return NULL;
  b2a_status s = b2a_kvcache_reset(c->cache, -1);
  if (s != B2A_OK) return throw_status(env, s);
  return undefined(env);
}

/* ---- the GPU model loop's per-layer dispatch (src/gpu/model.js:323-346) --------- */
typedef struct {
  b2a_rope* rope;
} Rope;

static void rope_finalize(napi_env env, void* data, void* hint) {
  (void)env;
  (void)hint;
  Rope* r = (Rope*)data;
  if (r->rope) b2a_rope_destroy(r->rope);
  free(r);
}

/* ropeCreate(headDim, theta, maxPositions) -> handle (the model's ropeTable, model.js:200-205) */
static napi_value RopeCreate(napi_env env, napi_callback_info info) {
  size_t argc = 3;
  napi_value argv[3], r;
  int32_t D, P;
  double theta;
  b2a_rope* rope = NULL;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  if (argc < 3 || !arg_int(env, argv[0], &D) || napi_get_value_double(env, argv[1], &theta) != napi_ok ||
      !arg_int(env, argv[2], &P)) {
    napi_throw_type_error(env, NULL, "ropeCreate(headDim, theta, maxPositions)");
    return NULL;
  }
  b2a_status s = b2a_rope_create(g_ctx, D, theta, P, &rope);
  if (s != B2A_OK) return throw_status(env, s);
  Rope* h = (Rope*)malloc(sizeof(Rope));
  if (h == NULL) {
    b2a_rope_destroy(rope);
    napi_throw_error(env, NULL, "out of host memory");
    return NULL;
  }
  h->rope = rope;
  napi_create_external(env, h, rope_finalize, NULL, &r);
  return r;
}

/* attentionDecode(cache, rope, layer, q, kNew, vNew, out, numHeads): RoPE(q), RoPE(k) + append at
 * the cache length, attention over length + 1 positions; f32 [numHeads*headDim] in and out.
 * The length is not advanced (commit after the last layer, as the reference does). */
static napi_value AttentionDecode(napi_env env, napi_callback_info info) {
  size_t argc = 8;
  napi_value argv[8];
  int32_t layer, H;
  void *q, *k, *v, *out;
  size_t n;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  Cache* c = argc >= 8 ? arg_cache(env, argv[0]) : NULL;
  void* rp = NULL;
  if (c == NULL || napi_get_value_external(env, argv[1], &rp) != napi_ok || rp == NULL ||
      !arg_int(env, argv[2], &layer) || !arg_typed(env, argv[3], napi_float32_array, &q, &n) ||
      !arg_typed(env, argv[4], napi_float32_array, &k, &n) || !arg_typed(env, argv[5], napi_float32_array, &v, &n) ||
      !arg_typed(env, argv[6], napi_float32_array, &out, &n) || !arg_int(env, argv[7], &H)) {
    return NULL;
  }
  b2a_status s = b2a_attention_decode(g_ctx, c->cache, ((Rope*)rp)->rope, layer, 1, H, q, k, v, B2A_F32, out,
                                      B2A_F32, B2A_HOST);
  if (s != B2A_OK) return throw_status(env, s);
  return argv[6];
}

/* attentionPrefill(cache, rope, layer, q, k, v, out, count, numHeads): `count` new tokens at the
 * cache length, causal, RoPE and append fused; f32 rows in and out. */
static napi_value AttentionPrefill(napi_env env, napi_callback_info info) {
  size_t argc = 9;
  napi_value argv[9];
  int32_t layer, count, H;
  void *q, *k, *v, *out;
  size_t n;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  Cache* c = argc >= 9 ? arg_cache(env, argv[0]) : NULL;
  void* rp = NULL;
  if (c == NULL || napi_get_value_external(env, argv[1], &rp) != napi_ok || rp == NULL ||
      !arg_int(env, argv[2], &layer) || !arg_typed(env, argv[3], napi_float32_array, &q, &n) ||
      !arg_typed(env, argv[4], napi_float32_array, &k, &n) || !arg_typed(env, argv[5], napi_float32_array, &v, &n) ||
      !arg_typed(env, argv[6], napi_float32_array, &out, &n) || !arg_int(env, argv[7], &count) ||
      !arg_int(env, argv[8], &H)) {
    return NULL;
  }
  b2a_status s = b2a_attention_prefill(g_ctx, c->cache, ((Rope*)rp)->rope, layer, 0, H, q, k, v, B2A_F32, count,
                                       out, B2A_F32, B2A_HOST);
  if (s != B2A_OK) return throw_status(env, s);
  return argv[6];
}

static void export_fn(napi_env env, napi_value exports, const char* name, napi_callback cb) {
  napi_value fn;
  napi_create_function(env, name, NAPI_AUTO_LENGTH, cb, NULL, &fn);
  napi_set_named_property(env, exports, name, fn);
}

/* The module's entry point (what NAPI_MODULE_INIT expands to). */
__attribute__((visibility("default"))) napi_value napi_register_module_v1(napi_env env, napi_value exports) {
  if (g_ctx == NULL && b2a_init(0, &g_ctx) != B2A_OK) {
    napi_throw_error(env, "B2A_ENODEV", b2a_last_error());
    return NULL;
  }
  export_fn(env, exports, "groupedAttention", GroupedAttention);
  export_fn(env, exports, "kvHeadFor", KvHeadFor);
  export_fn(env, exports, "ropeFrequencies", RopeFrequencies);
  export_fn(env, exports, "ropeTables", RopeTables);
  export_fn(env, exports, "kvCacheCreate", KvCacheCreate);
  export_fn(env, exports, "kvCacheAllocate", KvCacheAllocate);
  export_fn(env, exports, "kvCacheWriteAt", KvCacheWriteAt);
  export_fn(env, exports, "kvCacheKeysUpTo", KvCacheKeysUpTo);
  export_fn(env, exports, "kvCacheValuesUpTo", KvCacheValuesUpTo);
  export_fn(env, exports, "kvCachePresent", KvCachePresent);
  export_fn(env, exports, "kvCacheCommit", KvCacheCommit);
  export_fn(env, exports, "kvCacheLength", KvCacheLength);
  export_fn(env, exports, "kvCacheReset", KvCacheReset);
  export_fn(env, exports, "ropeCreate", RopeCreate);
  export_fn(env, exports, "attentionDecode", AttentionDecode);
  export_fn(env, exports, "attentionPrefill", AttentionPrefill);
  return exports;
}
