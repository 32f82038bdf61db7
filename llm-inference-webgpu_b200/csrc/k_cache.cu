// KV-cache kernels: fused RoPE(K) + round + append, raw writeAt, and the
// device mirror of the per-sequence lengths.
#include <climits>

#include "b2a_internal.cuh"
#include "k_util.cuh"

namespace b2a {

namespace {

// Eight 16-bit or f32 elements of a row -> f32 (vector loads when 16-byte aligned).
__device__ __forceinline__ void load8(const void* base, int64_t at, int dt, float (&x)[8]) {
  if (dt != DT_F32 && (reinterpret_cast<uintptr_t>(base) & 15) == 0) {
    const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + at);
    const uint16_t* hw = reinterpret_cast<const uint16_t*>(&u);
#pragma unroll
    for (int e = 0; e < 8; e++)
      x[e] = dt == DT_F16 ? __half2float(__ushort_as_half(hw[e])) : __bfloat162float(__ushort_as_bfloat16(hw[e]));
  } else if (dt == DT_F32 && (reinterpret_cast<uintptr_t>(base) & 15) == 0) {
    const float4* f4 = reinterpret_cast<const float4*>(static_cast<const float*>(base) + at);
    *reinterpret_cast<float4*>(&x[0]) = f4[0];
    *reinterpret_cast<float4*>(&x[4]) = f4[1];
  } else {
#pragma unroll
    for (int e = 0; e < 8; e++) x[e] = ld_as_f32(base, at + e, dt);
  }
}

// Eight f32 values -> a row of the cache dtype, rounded as st_from_f32 rounds
// (8-element rows of a 64-wide head are 16-byte aligned in the pools).
__device__ __forceinline__ void store8(void* base, int64_t at, int dt, const float (&x)[8]) {
  if (dt == DT_F32) {
    float4* f4 = reinterpret_cast<float4*>(static_cast<float*>(base) + at);
    f4[0] = make_float4(x[0], x[1], x[2], x[3]);
    f4[1] = make_float4(x[4], x[5], x[6], x[7]);
    return;
  }
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; e++) {
    const uint32_t lo = dt == DT_F16 ? f32_to_f16_bits(x[2 * e]) : f32_to_bf16_bits(x[2 * e]);
    const uint32_t hi = dt == DT_F16 ? f32_to_f16_bits(x[2 * e + 1]) : f32_to_bf16_bits(x[2 * e + 1]);
    w[e] = lo | (hi << 16);
  }
  *reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + at) = make_uint4(w[0], w[1], w[2], w[3]);
}

}  // namespace

// Query heads and KV heads one thread covers (the same 8 dims of one token in
// each): the rotation-table entries are loaded once for all of them, and the
// rows' loads are all in flight together.
constexpr int kQGroup = 2;
constexpr int kKVGroup = 1;

// src/cpu/model.js:103-116 (rope-k at absolute position past+t, then
// kv.writeAt), src/gpu/model.js:327-338 (ROPE on k, two copies), and, for the
// tensor-core prefill, RoPE(q) (src/cpu/model.js:103-106) as f16 rows.
// Grid (token blocks, sequences, head groups); a thread takes 8 dims (lane l:
// dims 8l..8l+7, 16 bytes of a 16-bit row) of one token in a group of heads,
// so eight neighbouring lanes cover a row (coalesced 16-byte accesses) and
// lanes l and l ^ 4 hold the two halves of each rotation pair, swapped by
// shuffle. Groups z < kv_groups rotate and append K and append V (kKVGroup KV
// heads per thread); the groups after them (when p.q_rot is set) rotate the
// queries (kQGroup heads per thread).
// K: IEEE f64 from the f64 table, every product and sum rounded separately
// (rope_pair_f64), then the cache dtype. Q: f32 from the f32 table, rounded
// once to f16, x[d] c - x[d+32] s and x[d+32] c + x[d] s: the arithmetic the
// prefill kernels' own query staging uses.
__global__ void __launch_bounds__(256, 5) k_rope_append(AttnParams p, int seq_first, int count, int kv_groups) {
  // a kernel launched after this one as a programmatic dependent may start its
  // prologue now; it waits for this grid before reading the cache
  asm volatile("griddepcontrol.launch_dependents;");
  const int b = static_cast<int>(blockIdx.y);
  const int seq_idx = seq_first + b;
  const int past = p.len[seq_idx];
  // grid z: the KV head groups, then the query head groups
  const bool kv = static_cast<int>(blockIdx.z) < kv_groups;
  const int heads = kv ? p.kv_heads : p.heads;
  const int h0 = (kv ? static_cast<int>(blockIdx.z) : static_cast<int>(blockIdx.z) - kv_groups) * (kv ? kKVGroup : kQGroup);
  const int i = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;   // 8 lanes per token
  const bool live = i < count * 8;
  const int ii = live ? i : 0;   // a lane past the end computes token 0 for the shuffles, stores nothing
  const int l = ii & 7;
  const int t = ii >> 3;
  const int pos = past + t;
  const int64_t row0 = (static_cast<int64_t>(b) * count + t) * heads;   // (sequence, token) row of head 0
  const int j0 = 8 * (l & 3);                                          // rotation index of the lane's first dim
  if (kv) {
    float x[kKVGroup][8], y[kKVGroup][8], vv[kKVGroup][8];
    uint4 vraw[kKVGroup];
    const bool vcopy = p.in_dtype == p.cache_dtype && p.cache_dtype != DT_F32 &&
                       (reinterpret_cast<uintptr_t>(p.v_new) & 15) == 0;   // the same 16-bit dtype: bits as given
#pragma unroll
    for (int m = 0; m < kKVGroup; m++) {
      const bool ok = live && h0 + m < heads;
      const int64_t at = (row0 + (ok ? h0 + m : 0)) * p.head_dim + 8 * l;
      load8(p.k_new, at, p.in_dtype, x[m]);
      if (vcopy) vraw[m] = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.v_new) + at);
      else load8(p.v_new, at, p.in_dtype, vv[m]);
    }
    // the lane's 8 table entries: 64 bytes at a 64-byte boundary of each table
    const double2* c2 = reinterpret_cast<const double2*>(p.rope_cos + static_cast<int64_t>(pos) * (p.head_dim / 2) + j0);
    const double2* s2 = reinterpret_cast<const double2*>(p.rope_sin + static_cast<int64_t>(pos) * (p.head_dim / 2) + j0);
    double cr[8], sr[8];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const double2 cc = c2[e], ss = s2[e];
      cr[2 * e] = cc.x;
      cr[2 * e + 1] = cc.y;
      sr[2 * e] = ss.x;
      sr[2 * e + 1] = ss.y;
    }
#pragma unroll
    for (int m = 0; m < kKVGroup; m++)
#pragma unroll
      for (int e = 0; e < 8; e++) y[m][e] = __shfl_xor_sync(0xffffffffu, x[m][e], 4);
#pragma unroll
    for (int m = 0; m < kKVGroup; m++) {
      if (!live || h0 + m >= heads) continue;
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const double dx = static_cast<double>(x[m][e]), dy = static_cast<double>(y[m][e]);
        // first half (l < 4): lo c - hi s; second half: hi c + lo s
        o[e] = l < 4 ? __double2float_rn(__dsub_rn(__dmul_rn(dx, cr[e]), __dmul_rn(dy, sr[e])))
                     : __double2float_rn(__dadd_rn(__dmul_rn(dx, cr[e]), __dmul_rn(dy, sr[e])));
      }
      const int64_t dst = kv_elem(p, seq_idx, p.layer_begin, h0 + m, pos) + 8 * l;
      store8(p.kc_w, dst, p.cache_dtype, o);
      if (vcopy) *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.vc_w) + dst) = vraw[m];
      else store8(p.vc_w, dst, p.cache_dtype, vv[m]);   // exact when the dtypes agree, else rounded as st_from_f32
    }
  } else {
    float x[kQGroup][8];
#pragma unroll
    for (int m = 0; m < kQGroup; m++) {
      const bool ok = live && h0 + m < heads;
      load8(p.q, (row0 + (ok ? h0 + m : 0)) * p.head_dim + 8 * l, p.in_dtype, x[m]);
    }
    const int64_t ra = static_cast<int64_t>(pos) * (p.head_dim / 2) + j0;
    float c[8], sn[8];
    *reinterpret_cast<float4*>(&c[0]) = *reinterpret_cast<const float4*>(p.rope_cos32 + ra);
    *reinterpret_cast<float4*>(&c[4]) = *reinterpret_cast<const float4*>(p.rope_cos32 + ra + 4);
    *reinterpret_cast<float4*>(&sn[0]) = *reinterpret_cast<const float4*>(p.rope_sin32 + ra);
    *reinterpret_cast<float4*>(&sn[4]) = *reinterpret_cast<const float4*>(p.rope_sin32 + ra + 4);
    // first half (l < 4): x c - y s, second half: x c + y s, as x c + y (-/+ s)
    // (a sign flip is exact, so the product rounds as y s would)
    if (l < 4) {
#pragma unroll
      for (int e = 0; e < 8; e++) sn[e] = -sn[e];
    }
#pragma unroll
    for (int m = 0; m < kQGroup; m++) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float y0 = __shfl_xor_sync(0xffffffffu, x[m][e], 4);
        const float y1 = __shfl_xor_sync(0xffffffffu, x[m][e + 1], 4);
        const __half2 h2 = __floats2half2_rn(fmaf(x[m][e], c[e], y0 * sn[e]), fmaf(x[m][e + 1], c[e + 1], y1 * sn[e + 1]));
        w[e >> 1] = *reinterpret_cast<const uint32_t*>(&h2);
      }
      if (live && h0 + m < heads) {
        *reinterpret_cast<uint4*>(p.q_rot + (row0 + h0 + m) * p.head_dim + 8 * l) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
}

cudaError_t launch_rope_append(const AttnParams& p, int seq_idx, int count, cudaStream_t st, int nseq) {
  if (count <= 0 || nseq <= 0) return cudaSuccess;
  if (p.head_dim != 64 || nseq > 65535) return cudaErrorInvalidValue;
  const int threads = 256;
  const int64_t lanes = static_cast<int64_t>(count) * 8;   // per (sequence, head group)
  if (lanes > INT32_MAX - threads) return cudaErrorInvalidValue;
  const int kv_groups = (p.kv_heads + kKVGroup - 1) / kKVGroup;
  const int q_groups = p.q_rot != nullptr ? (p.heads + kQGroup - 1) / kQGroup : 0;
  const int blocks = static_cast<int>((lanes + threads - 1) / threads);
  k_rope_append<<<dim3(blocks, nseq, kv_groups + q_groups), threads, 0, st>>>(p, seq_idx, count, kv_groups);
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
