// KV-cache kernels: fused RoPE(K) + round + append, raw writeAt, and the
// device mirror of the per-sequence lengths.
#include "b2a_internal.cuh"
#include "k_util.cuh"

namespace b2a {

// src/cpu/model.js:103-116 (rope-k at absolute position past+t, then
// kv.writeAt), src/gpu/model.js:327-338 (ROPE on k, two copies). One thread
// per rotation pair (t, kv head, j); the same thread stores both halves of V.
__global__ void k_rope_append(AttnParams p, int seq_first, int count, int nseq) {
  // a kernel launched after this one as a programmatic dependent may start its
  // prologue now; it waits for this grid before reading the cache
  asm volatile("griddepcontrol.launch_dependents;");
  const int half = p.head_dim >> 1;
  const int64_t n = static_cast<int64_t>(count) * p.kv_heads * half;   // per sequence
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n * nseq;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(i / n);
    const int64_t ib = i - b * n;
    const int seq_idx = seq_first + b;
    const int past = p.len[seq_idx];
    const int j = static_cast<int>(ib % half);
    const int g = static_cast<int>((ib / half) % p.kv_heads);
    const int t = static_cast<int>(ib / (static_cast<int64_t>(half) * p.kv_heads));
    const int pos = past + t;
    const int64_t src = ((static_cast<int64_t>(b) * count + t) * p.kv_heads + g) * p.head_dim;
    const int64_t dst = kv_elem(p, seq_idx, p.layer_begin, g, pos);
    const double c = p.rope_cos[static_cast<int64_t>(pos) * half + j];
    const double s = p.rope_sin[static_cast<int64_t>(pos) * half + j];
    float lo, hi;
    rope_pair_f64(ld_as_f32(p.k_new, src + j, p.in_dtype), ld_as_f32(p.k_new, src + j + half, p.in_dtype), c,
                  s, lo, hi);
    st_from_f32(p.kc_w, dst + j, p.cache_dtype, lo);
    st_from_f32(p.kc_w, dst + j + half, p.cache_dtype, hi);
    convert_elem(p.v_new, src + j, p.in_dtype, p.vc_w, dst + j, p.cache_dtype);
    convert_elem(p.v_new, src + j + half, p.in_dtype, p.vc_w, dst + j + half, p.cache_dtype);
  }
}

cudaError_t launch_rope_append(const AttnParams& p, int seq_idx, int count, cudaStream_t st, int nseq) {
  const int64_t n = static_cast<int64_t>(count) * p.kv_heads * (p.head_dim / 2) * nseq;
  if (n == 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = static_cast<int>((n + threads - 1) / threads < 4096 ? (n + threads - 1) / threads : 4096);
  k_rope_append<<<blocks, threads, 0, st>>>(p, seq_idx, count, nseq);
  return cudaGetLastError();
}

// src/cpu/cache.js:63-67: rows [count][kv_heads*head_dim] stored as given
// (rounded to the cache dtype) at positions at..at+count-1, head-major.
__global__ void k_write_at(AttnParams p, int seq_idx, int layer, const void* k, const void* v, int src_dt, int count,
                           int at) {
  const int64_t n = static_cast<int64_t>(count) * p.kv_heads * p.head_dim;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int d = static_cast<int>(i % p.head_dim);
    const int g = static_cast<int>((i / p.head_dim) % p.kv_heads);
    const int t = static_cast<int>(i / (static_cast<int64_t>(p.head_dim) * p.kv_heads));
    const int64_t dst = kv_elem(p, seq_idx, layer, g, at + t) + d;
    convert_elem(k, i, src_dt, p.kc_w, dst, p.cache_dtype);
    convert_elem(v, i, src_dt, p.vc_w, dst, p.cache_dtype);
  }
}

void fill_cache_params(AttnParams& p, const b2a_kvcache* c) {
  p.kc = c->d_k;
  p.vc = c->d_v;
  p.kc_w = c->d_k;
  p.vc_w = c->d_v;
  p.s_seq = c->s_seq;
  p.s_layer = c->s_layer;
  p.s_head = c->s_head;
  p.pages = c->page_size > 0 ? c->d_pages : nullptr;
  p.max_pages = c->max_pages;
  p.page_shift = c->page_shift;
  p.cache_dtype = static_cast<int>(c->dtype);
  p.len = c->d_len;
  p.kv_heads = c->kv_heads;
  p.head_dim = c->head_dim;
}

cudaError_t launch_write_at(const b2a_kvcache* c, int layer, int seq_idx, int at, const void* k, const void* v,
                            int src_dtype, int count, cudaStream_t st) {
  const int64_t n = static_cast<int64_t>(count) * c->kv_heads * c->head_dim;
  if (n == 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = static_cast<int>((n + threads - 1) / threads < 4096 ? (n + threads - 1) / threads : 4096);
  AttnParams p{};
  fill_cache_params(p, c);
  k_write_at<<<blocks, threads, 0, st>>>(p, seq_idx, layer, k, v, src_dtype, count, at);
  return cudaGetLastError();
}

// mode 0: len[idx] += count (idx < 0: every sequence); mode 1: len[idx] = 0
// (idx < 0: every sequence). Keeps the device lengths in stream order with the
// host's bookkeeping.
__global__ void k_lengths_update(int32_t* len, int idx, int batch, int count, int mode) {
  for (int b = threadIdx.x + blockIdx.x * blockDim.x; b < batch; b += blockDim.x * gridDim.x) {
    if (idx >= 0 && b != idx) continue;
    if (mode == 0) len[b] += count;
    else len[b] = 0;
  }
}

cudaError_t launch_lengths_update(int32_t* d_len, int idx, int batch, int count, int mode, cudaStream_t st) {
  const int threads = 256;
  const int blocks = (batch + threads - 1) / threads;
  k_lengths_update<<<blocks > 0 ? blocks : 1, threads, 0, st>>>(d_len, idx, batch, count, mode);
  return cudaGetLastError();
}

}  // namespace b2a
