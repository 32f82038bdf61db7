// CUDA-core attention kernels:
//  - k_attn_simt: split-KV attention over the head-major cache, any cache
//    dtype, one CTA per (query row group, KV chunk). It serves f32 caches and
//    every shape the tensor-core kernels do not.
//  - k_combine: log-sum-exp merge of split-KV partials.
//  - k_grouped_generic: the literal groupedAttention drop-in over
//    position-major f32 arrays (src/core/attention.js:32-66), any head layout.
#include <math_constants.h>

#include "b2a_internal.cuh"
#include "k_util.cuh"

namespace b2a {

namespace {
constexpr int kSimtThreads = 128;
constexpr int kSimtMaxGroup = 8;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
}  // namespace

// One CTA: one (sequence b, layer, token t, KV head g) row group of `group`
// query heads, over KV positions [c*chunk, min((c+1)*chunk, n_keys)).
// Writes the unnormalised partial (o, m, l) per query head, base-2 units.
template <int D>
__global__ void __launch_bounds__(kSimtThreads) k_attn_simt(AttnParams p) {
  constexpr int half = D / 2;
  __shared__ float qs[kSimtMaxGroup][D];
  __shared__ float sc[kSimtMaxGroup][256];
  __shared__ float red[kSimtMaxGroup][D];
  __shared__ float sm_m[kSimtMaxGroup], sm_l[kSimtMaxGroup];

  const int tid = threadIdx.x;
  const int G = p.group;
  int r = blockIdx.x;
  const int g = r % p.kv_heads;
  r /= p.kv_heads;
  const int t = r % p.tokens;
  r /= p.tokens;
  const int l = r % p.num_layers;
  const int b = r / p.num_layers;          // relative to this call
  const int bc = p.seq_begin + b;          // cache sequence
  const int c = blockIdx.y;

  const int past = p.len[bc];
  const int pos_q = (p.q_pos ? p.q_pos[b] : past) + t;   // absolute RoPE position of this token
  const int slot = past + t;                               // cache position of this token
  const int n_keys = past + t + p.horizon_extra;
  const int p0 = c * p.chunk;
  const int p1 = min(p0 + p.chunk, n_keys);
  const int64_t row0 = ((static_cast<int64_t>(b) * p.num_layers + l) * p.tokens + t) * p.heads + g * G;
  float* part = p.partial + (row0 * p.nchunks + c) * (D + 4);
  const int64_t part_row = static_cast<int64_t>(p.nchunks) * (D + 4);

  if (p0 >= n_keys) {   // empty chunk of a shorter row: contributes nothing
    for (int i = tid; i < G; i += blockDim.x) {
      part[i * part_row + D] = -CUDART_INF_F;
      part[i * part_row + D + 1] = 0.f;
    }
    return;
  }

  const int layer = p.layer_begin + l;
  const int64_t cache_base = kv_elem(p, bc, layer, g, 0);   // position 0 (contiguous: the row base)
  const double* cosr = p.rope_cos + static_cast<int64_t>(pos_q) * half;
  const double* sinr = p.rope_sin + static_cast<int64_t>(pos_q) * half;

  // RoPE(q) for the group's heads (src/core/ops.js:147-158), f64 -> f32.
  const int64_t qrow = row0 * D;
  for (int i = tid; i < G * half; i += blockDim.x) {
    const int h = i / half, j = i % half;
    float lo, hi;
    rope_pair_f64(ld_as_f32(p.q, qrow + h * D + j, p.in_dtype), ld_as_f32(p.q, qrow + h * D + j + half, p.in_dtype),
                  cosr[j], sinr[j], lo, hi);
    qs[h][j] = lo;
    qs[h][j + half] = hi;
  }
  // Fused append of this token's key/value (single-token rows only), by the
  // one CTA whose chunk holds the new slot.
  if (p.k_new != nullptr && slot >= p0 && slot < p1) {
    const int64_t src = (((static_cast<int64_t>(b) * p.num_layers + l) * p.tokens + t) * p.kv_heads + g) * D;
    const int64_t dst = kv_elem(p, bc, layer, g, slot);
    for (int j = tid; j < half; j += blockDim.x) {
      float lo, hi;
      rope_pair_f64(ld_as_f32(p.k_new, src + j, p.in_dtype), ld_as_f32(p.k_new, src + j + half, p.in_dtype),
                    cosr[j], sinr[j], lo, hi);
      st_from_f32(p.kc_w, dst + j, p.cache_dtype, lo);
      st_from_f32(p.kc_w, dst + j + half, p.cache_dtype, hi);
      convert_elem(p.v_new, src + j, p.in_dtype, p.vc_w, dst + j, p.cache_dtype);
      convert_elem(p.v_new, src + j + half, p.in_dtype, p.vc_w, dst + j + half, p.cache_dtype);
    }
  }
  __syncthreads();

  const float scale2 = rsqrtf(static_cast<float>(D)) * kLog2e;
  const int n = p1 - p0;
  // scores: thread i takes positions i and i+128 of the chunk
  for (int i = tid; i < n; i += blockDim.x) {
    const int64_t krow = p.pages ? kv_elem(p, bc, layer, g, p0 + i) : cache_base + static_cast<int64_t>(p0 + i) * D;
    float acc[kSimtMaxGroup];
#pragma unroll
    for (int h = 0; h < kSimtMaxGroup; h++) acc[h] = 0.f;
    for (int d = 0; d < D; d++) {
      const float kv = ld_as_f32(p.kc, krow + d, p.cache_dtype);
#pragma unroll
      for (int h = 0; h < kSimtMaxGroup; h++)
        if (h < G) acc[h] = fmaf(qs[h][d], kv, acc[h]);
    }
#pragma unroll
    for (int h = 0; h < kSimtMaxGroup; h++)
      if (h < G) sc[h][i] = acc[h] * scale2;
  }
  __syncthreads();

  // per-head max and exponentials (one warp per head)
  const int warp = tid >> 5, lane = tid & 31;
  for (int h = warp; h < G; h += blockDim.x / 32) {
    float m = -CUDART_INF_F;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, sc[h][i]);
    m = warp_max(m);
    float s = 0.f;
    for (int i = lane; i < n; i += 32) {
      const float e = exp2f(sc[h][i] - m);
      sc[h][i] = e;
      s += e;
    }
    s = warp_sum(s);
    if (lane == 0) { sm_m[h] = m; sm_l[h] = s; }
  }
  __syncthreads();

  // PV: thread (hf, d) sums every other position of the chunk
  const int d = tid % D;
  const int hf = tid / D;
  const int nhalves = blockDim.x / D;
  float acc[kSimtMaxGroup];
#pragma unroll
  for (int h = 0; h < kSimtMaxGroup; h++) acc[h] = 0.f;
  for (int i = hf; i < n; i += nhalves) {
    const int64_t vrow = p.pages ? kv_elem(p, bc, layer, g, p0 + i) : cache_base + static_cast<int64_t>(p0 + i) * D;
    const float vv = ld_as_f32(p.vc, vrow + d, p.cache_dtype);
#pragma unroll
    for (int h = 0; h < kSimtMaxGroup; h++)
      if (h < G) acc[h] = fmaf(sc[h][i], vv, acc[h]);
  }
  for (int step = 1; step < nhalves; step++) {
    if (hf == step) {
      for (int h = 0; h < G; h++) red[h][d] = acc[h];
    }
    __syncthreads();
    if (hf == 0) {
      for (int h = 0; h < G; h++) acc[h] += red[h][d];
    }
    __syncthreads();
  }
  if (hf == 0) {
    for (int h = 0; h < G; h++) part[h * part_row + d] = acc[h];
  }
  if (tid < G) {
    part[tid * part_row + D] = sm_m[tid];
    part[tid * part_row + D + 1] = sm_l[tid];
  }
}

cudaError_t launch_attn_simt(const AttnParams& p, cudaStream_t st) {
  if (p.head_dim != 64 || p.group > kSimtMaxGroup || p.chunk > 256) return cudaErrorInvalidValue;
  const int64_t groups = static_cast<int64_t>(p.batch) * p.num_layers * p.tokens * p.kv_heads;
  if (groups == 0 || p.nchunks == 0) return cudaSuccess;
  if (groups > 0x7fffffff || p.nchunks > 65535) return cudaErrorInvalidValue;
  dim3 grid(static_cast<unsigned>(groups), static_cast<unsigned>(p.nchunks));
  k_attn_simt<64><<<grid, kSimtThreads, 0, st>>>(p);
  return cudaGetLastError();
}

// One warp per output row (b, layer, t, head): merge the row's partials in
// ascending order. m* = max m_i, w_i = 2^(m_i - m*), out = sum w_i o_i / sum w_i l_i.
__global__ void k_combine(CombineParams p, int64_t row_stride, int64_t part_stride) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int D = p.head_dim;
  if (row >= p.rows) return;
  int parts = p.nchunks;
  if (p.len != nullptr) {   // chunks this row actually wrote
    int64_t r = row / p.heads;
    const int t = static_cast<int>(r % p.tokens);
    r /= p.tokens;
    const int b = static_cast<int>(r / p.num_layers);
    const int nk = p.len[p.seq_begin + b] + t + p.extra;
    parts = nk > 0 ? (nk + p.chunk - 1) / p.chunk : 1;
    if (parts > p.nchunks) parts = p.nchunks;
  }
  const float* base = p.partial + row * row_stride;
  float m = -CUDART_INF_F;
  for (int i = 0; i < parts; i++) {
    const float* pp = base + i * part_stride;
    if (pp[D + 1] > 0.f) m = fmaxf(m, pp[D]);
  }
  float lsum = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};   // D <= 128
  for (int i = 0; i < parts; i++) {
    const float* pp = base + i * part_stride;
    const float li = pp[D + 1];
    if (!(li > 0.f)) continue;
    const float w = exp2f(pp[D] - m);
    lsum = fmaf(w, li, lsum);
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int d = lane + 32 * k;
      if (d < D) acc[k] = fmaf(w, pp[d], acc[k]);
    }
  }
  if (p.mode == 1) {   // merged partial: o and l rescaled to the common max m
    float* o = static_cast<float*>(p.out) + row * (D + 4);
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int d = lane + 32 * k;
      if (d < D) o[d] = acc[k];
    }
    if (lane == 0) { o[D] = m; o[D + 1] = lsum; o[D + 2] = 0.f; o[D + 3] = 0.f; }
    return;
  }
  const float inv = 1.f / lsum;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int d = lane + 32 * k;
    if (d < D) st_from_f32(p.out, row * D + d, p.out_dtype, acc[k] * inv);
  }
}

// Rows with many partials (long contexts split into many chunks): one CTA per
// row, each of its 8 warps merges every 8th partial with an online rescale,
// then warp 0 merges the 8 results in warp order (a fixed order: the same
// inputs always give the same bits).
__global__ void __launch_bounds__(256) k_combine_wide(CombineParams p, int64_t row_stride, int64_t part_stride) {
  __shared__ float sm_m[8], sm_l[8], sm_o[8][128];
  const int64_t row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = p.head_dim;
  int parts = p.nchunks;
  if (p.len != nullptr) {
    int64_t r = row / p.heads;
    const int t = static_cast<int>(r % p.tokens);
    r /= p.tokens;
    const int b = static_cast<int>(r / p.num_layers);
    const int nk = p.len[p.seq_begin + b] + t + p.extra;
    parts = nk > 0 ? (nk + p.chunk - 1) / p.chunk : 1;
    if (parts > p.nchunks) parts = p.nchunks;
  }
  const float* base = p.partial + row * row_stride;
  // this warp's parts are i = warp + 8 k; lane k holds part k's (m, l), so one
  // load instruction fetches up to 32 of them, and the weighted sum below
  // issues its loads independently of each other
  float m = -CUDART_INF_F, lsum = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; warp + 8 * k0 < parts; k0 += 32) {
    const int i = warp + 8 * (k0 + lane);
    float mi = -CUDART_INF_F, li = 0.f;
    if (i < parts) {
      const float* pp = base + i * part_stride;
      mi = pp[D];
      li = pp[D + 1];
      if (!(li > 0.f)) mi = -CUDART_INF_F;
    }
    float mx = mi;
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float mn = fmaxf(m, mx);
    if (mn == -CUDART_INF_F) continue;
    const float a = (m == -CUDART_INF_F) ? 0.f : exp2f(m - mn);
    const float wi = (mi == -CUDART_INF_F) ? 0.f : exp2f(mi - mn);
    float lw = wi * li;
    for (int o = 16; o > 0; o >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, o);
    lsum = fmaf(lsum, a, lw);
#pragma unroll
    for (int k = 0; k < 4; k++) acc[k] *= a;
    const int nk = min(32, (parts - warp + 7) / 8 - k0);
#pragma unroll 4
    for (int kk = 0; kk < nk; kk++) {
      const float w = __shfl_sync(0xffffffffu, wi, kk);
      const float* pp = base + (warp + 8 * (k0 + kk)) * part_stride;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int d = lane + 32 * k;
        if (d < D) acc[k] = fmaf(w, pp[d], acc[k]);
      }
    }
    m = mn;
  }
  if (lane == 0) {
    sm_m[warp] = m;
    sm_l[warp] = lsum;
  }
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int d = lane + 32 * k;
    if (d < D) sm_o[warp][d] = acc[k];
  }
  __syncthreads();
  if (warp != 0) return;
  float mx = -CUDART_INF_F;
  for (int w = 0; w < 8; w++)
    if (sm_l[w] > 0.f) mx = fmaxf(mx, sm_m[w]);
  float L = 0.f;
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  for (int w = 0; w < 8; w++) {
    if (!(sm_l[w] > 0.f)) continue;
    const float s = exp2f(sm_m[w] - mx);
    L = fmaf(s, sm_l[w], L);
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int d = lane + 32 * k;
      if (d < D) o[k] = fmaf(s, sm_o[w][d], o[k]);
    }
  }
  if (p.mode == 1) {
    float* out = static_cast<float*>(p.out) + row * (D + 4);
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int d = lane + 32 * k;
      if (d < D) out[d] = o[k];
    }
    if (lane == 0) { out[D] = mx; out[D + 1] = L; out[D + 2] = 0.f; out[D + 3] = 0.f; }
    return;
  }
  const float inv = 1.f / L;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int d = lane + 32 * k;
    if (d < D) st_from_f32(p.out, row * D + d, p.out_dtype, o[k] * inv);
  }
}

cudaError_t launch_combine(const CombineParams& p, cudaStream_t st) {
  if (p.head_dim > 128) return cudaErrorInvalidValue;
  if (p.rows == 0) return cudaSuccess;
  const int64_t stride_part = p.part_stride_rows ? static_cast<int64_t>(p.part_stride_rows) * (p.head_dim + 4)
                                                 : (p.head_dim + 4);
  const int64_t stride_row = p.part_stride_rows ? (p.head_dim + 4)
                                                : static_cast<int64_t>(p.nchunks) * (p.head_dim + 4);
  if (p.nchunks >= 16) {
    k_combine_wide<<<static_cast<unsigned>(p.rows), 256, 0, st>>>(p, stride_row, stride_part);
    return cudaGetLastError();
  }
  const int threads = 256;
  const int64_t blocks = (static_cast<int64_t>(p.rows) * 32 + threads - 1) / threads;
  k_combine<<<static_cast<unsigned>(blocks), threads, 0, st>>>(p, stride_row, stride_part);
  return cudaGetLastError();
}

// Loads the CUDA-core decode and the combine kernels onto the current device
// (otherwise loaded lazily at their first launch, which allocates device memory).
cudaError_t preload_attn_simt() {
  cudaFuncAttributes a;
  cudaError_t e = cudaFuncGetAttributes(&a, k_attn_simt<64>);
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, k_combine);
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, k_combine_wide);
  return e;
}

// src/core/attention.js:32-66 over position-major f32 arrays, any head layout,
// head_dim <= 256. One CTA per (query t, head h); keys are walked in chunks of
// 1024 with an online (rescaled) softmax so any context length fits.
__global__ void __launch_bounds__(256) k_grouped_generic(const float* q, const float* keys, const float* values,
                                                         float* out, int seq, int past, int H, int KVH, int D) {
  constexpr int CH = 1024;
  __shared__ float qs[256];
  __shared__ float sc[CH];
  __shared__ float red[32];
  const int t = blockIdx.x / H, h = blockIdx.x % H;
  const int G = H / KVH;
  const int q_dim = H * D, kv_dim = KVH * D;
  const int kvb = (h / G) * D;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  for (int d = tid; d < D; d += blockDim.x) qs[d] = q[static_cast<int64_t>(t) * q_dim + h * D + d];
  __syncthreads();
  const float scale2 = rsqrtf(static_cast<float>(D)) * kLog2e;
  const int n = past + t + 1;
  float m = -CUDART_INF_F, lsum = 0.f, acc = 0.f;
  for (int c0 = 0; c0 < n; c0 += CH) {
    const int cn = min(CH, n - c0);
    float lmax = -CUDART_INF_F;
    for (int i = tid; i < cn; i += blockDim.x) {
      const float* kr = keys + static_cast<int64_t>(c0 + i) * kv_dim + kvb;
      float dot = 0.f;
      for (int d = 0; d < D; d++) dot = fmaf(qs[d], kr[d], dot);
      sc[i] = dot * scale2;
      lmax = fmaxf(lmax, sc[i]);
    }
    lmax = warp_max(lmax);
    if (lane == 0) red[warp] = lmax;
    __syncthreads();
    float cmax = -CUDART_INF_F;
    for (int w = 0; w < nw; w++) cmax = fmaxf(cmax, red[w]);
    const float m_new = fmaxf(m, cmax);
    const float alpha = exp2f(m - m_new);
    __syncthreads();
    float ls = 0.f;
    for (int i = tid; i < cn; i += blockDim.x) {
      const float e = exp2f(sc[i] - m_new);
      sc[i] = e;
      ls += e;
    }
    ls = warp_sum(ls);
    if (lane == 0) red[warp] = ls;
    __syncthreads();
    float csum = 0.f;
    for (int w = 0; w < nw; w++) csum += red[w];
    lsum = lsum * alpha + csum;
    if (tid < D) {
      float a = acc * alpha;
      const float* vr = values + static_cast<int64_t>(c0) * kv_dim + kvb + tid;
      for (int i = 0; i < cn; i++) a = fmaf(sc[i], vr[static_cast<int64_t>(i) * kv_dim], a);
      acc = a;
    }
    m = m_new;
    __syncthreads();
  }
  if (tid < D) out[static_cast<int64_t>(t) * q_dim + h * D + tid] = acc / lsum;
}

cudaError_t launch_grouped_generic(const float* q, const float* k, const float* v, float* out, int seq, int past,
                                   int heads, int kv_heads, int head_dim, cudaStream_t st) {
  if (head_dim > 256) return cudaErrorInvalidValue;
  const int64_t blocks = static_cast<int64_t>(seq) * heads;
  if (blocks == 0) return cudaSuccess;
  k_grouped_generic<<<static_cast<unsigned>(blocks), 256, 0, st>>>(q, k, v, out, seq, past, heads, kv_heads,
                                                                    head_dim);
  return cudaGetLastError();
}

}  // namespace b2a
