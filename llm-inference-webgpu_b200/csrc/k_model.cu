// The decoder's small kernels around attention and the projections: the
// embedding lookup, RMSNorm, SwiGLU and the greedy argmax
// (src/cpu/model.js:55-187 with src/core/ops.js:17-24, 81-91).
//
// Each is a single pass over at most a few MB (the argmax reads the 608 KB of
// logits, the rest read one or a few rows), so they are latency-bound; what
// matters is one launch each and no dependent global round trips. They keep
// the reference's f64 arithmetic (its JS numbers) where it has it: the norm's
// sum of squares and scale, and silu. All of them are launched as programmatic
// dependents and read nothing before griddepcontrol.wait.
#include <algorithm>
#include <cfloat>
#include <climits>

#include "b2a_internal.cuh"
#include "k_util.cuh"

namespace b2a {

namespace {

__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <typename Kernel, typename... Args>
cudaError_t launch_pdl(Kernel k, dim3 grid, dim3 block, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

constexpr int kNormThreads = 256;
constexpr int kArgThreads = 256;
constexpr int kArgMaxCtas = 512;

}  // namespace

// One token per CTA: x[t][i] = code * scale, the dequantized row
// (src/core/quantize.js:60-67; the lookup itself is src/cpu/model.js:195-210).
// An id outside [0, vocab) sets kErrBadToken and leaves the row zero.
__global__ void __launch_bounds__(256) k_embed_int8(const int32_t* tokens, const int8_t* codes, const void* scales,
                                                    int scale_dtype, int hidden, int vocab, float* x, int32_t* err) {
  pdl_enter();
  const int t = blockIdx.x;
  const int id = tokens[t];
  float* row = x + static_cast<int64_t>(t) * hidden;
  if (id < 0 || id >= vocab) {
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) row[i] = 0.f;
    if (threadIdx.x == 0) atomicOr(err, kErrBadToken);
    return;
  }
  const float s = ld_as_f32(scales, id, scale_dtype);
  const char4* src = reinterpret_cast<const char4*>(codes + static_cast<int64_t>(id) * hidden);
  for (int i = threadIdx.x; i < hidden / 4; i += blockDim.x) {
    const char4 c = src[i];
    // an int8 times an f32 is exact in f64, so the f32 product is the
    // correctly rounded one the reference stores
    reinterpret_cast<float4*>(row)[i] =
        make_float4(static_cast<float>(c.x) * s, static_cast<float>(c.y) * s, static_cast<float>(c.z) * s,
                    static_cast<float>(c.w) * s);
  }
}

// One row per CTA (src/core/ops.js:17-24): the sum of squares in f64 (each
// f32 square is exact in f64; only the order of the f64 additions differs
// from the reference's), scale = 1 / sqrt(ss / n + eps) in f64, and
// out = (x * scale) * w rounded once to f32.
__global__ void __launch_bounds__(kNormThreads) k_rmsnorm(const float* x, const float* w, double eps, int hidden,
                                                          float* out) {
  pdl_enter();
  __shared__ double red[kNormThreads / 32];
  __shared__ double s_scale;
  const float* row = x + static_cast<int64_t>(blockIdx.x) * hidden;
  float* orow = out + static_cast<int64_t>(blockIdx.x) * hidden;
  double ss = 0.0;
  for (int i = threadIdx.x; i < hidden; i += kNormThreads) {
    const double v = row[i];
    ss = __dadd_rn(ss, __dmul_rn(v, v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; i++) t = __dadd_rn(t, red[i]);
    s_scale = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(t, static_cast<double>(hidden)), eps)));
  }
  __syncthreads();
  const double scale = s_scale;
  for (int i = threadIdx.x; i < hidden; i += kNormThreads) {
    orow[i] = __double2float_rn(__dmul_rn(__dmul_rn(static_cast<double>(row[i]), scale), static_cast<double>(w[i])));
  }
}

// h[i] = silu(gu[2i]) * gu[2i+1] (gate and up outputs interleaved), silu(g) =
// g / (1 + exp(-g)) in f64 (src/core/ops.js:81-91), stored f32.
__global__ void __launch_bounds__(256) k_swiglu(const float* gu, float* h, int64_t n) {
  pdl_enter();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float2 v = reinterpret_cast<const float2*>(gu)[i];
    const double g = v.x;
    const double s = __ddiv_rn(g, __dadd_rn(1.0, exp(-g)));
    h[i] = __double2float_rn(__dmul_rn(s, static_cast<double>(v.y)));
  }
}

namespace {
// (value, index) order of the greedy pick: larger value first, then the
// smaller index (the reference keeps the first maximum, model.js:182-183)
__device__ __forceinline__ bool arg_better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}
}  // namespace

// The greedy pick over logits[0..n): each CTA reduces a contiguous stretch to
// its first maximum, the last CTA to finish (a counter in scratch) reduces the
// CTAs' results in order and writes the token. NaNs never win, as with the
// reference's `>`; when nothing beats logits[0] (a NaN or -inf there, or every
// value -inf) the token is 0 as in the reference.
__global__ void __launch_bounds__(kArgThreads) k_argmax(const float* logits, int n, int per_cta, int32_t* token,
                                                        float* value, float* part_v, int32_t* part_i,
                                                        uint32_t* counter) {
  pdl_enter();
  __shared__ float sv[kArgThreads / 32];
  __shared__ int si[kArgThreads / 32];
  __shared__ bool last;
  const int begin = blockIdx.x * per_cta, end = min(n, begin + per_cta);
  float bv = -INFINITY;
  int bi = INT_MAX;
  for (int i = begin + threadIdx.x; i < end; i += kArgThreads) {
    const float v = logits[i];
    if (v > bv) {   // ascending indices per thread: strict > keeps the first
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (arg_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kArgThreads / 32; w++) {
      if (arg_better(sv[w], si[w], bv, bi)) {
        bv = sv[w];
        bi = si[w];
      }
    }
    part_v[blockIdx.x] = bv;
    part_i[blockIdx.x] = bi;
    __threadfence();
    last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  bv = -INFINITY;
  bi = INT_MAX;
  for (int c = 0; c < static_cast<int>(gridDim.x); c++) {
    const float v = __ldcg(part_v + c);
    const int i = __ldcg(part_i + c);
    if (arg_better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  const float l0 = logits[0];
  if (bi == INT_MAX || !(bv > l0)) {   // nothing beats logits[0]
    bi = 0;
    bv = l0;
  }
  *token = bi;
  if (value) *value = bv;
  *counter = 0u;
}

cudaError_t launch_embed_int8(const int32_t* tokens, int count, const int8_t* codes, const void* scales,
                              int scale_dtype, int hidden, int vocab, float* x, int32_t* err, cudaStream_t st) {
  if (count <= 0) return cudaSuccess;
  if (hidden % 4 != 0) return cudaErrorInvalidValue;
  return launch_pdl(k_embed_int8, dim3(count), dim3(256), st, tokens, codes, scales, scale_dtype, hidden, vocab, x,
                    err);
}

cudaError_t launch_rmsnorm(const float* x, const float* w, double eps, int rows, int hidden, float* out,
                           cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  return launch_pdl(k_rmsnorm, dim3(rows), dim3(kNormThreads), st, x, w, eps, hidden, out);
}

cudaError_t launch_swiglu(const float* gu, float* h, int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 8);
  return launch_pdl(k_swiglu, dim3(static_cast<unsigned>(blocks)), dim3(256), st, gu, h, n);
}

cudaError_t launch_argmax(const float* logits, int n, int32_t* token, float* value, void* scratch,
                          cudaStream_t st) {
  if (n <= 0) return cudaErrorInvalidValue;
  // a stretch of at least 4 values per thread, at most kArgMaxCtas CTAs
  int ctas = (n + 4 * kArgThreads - 1) / (4 * kArgThreads);
  ctas = std::max(1, std::min(ctas, kArgMaxCtas));
  const int per_cta = (n + ctas - 1) / ctas;
  ctas = (n + per_cta - 1) / per_cta;
  auto* base = static_cast<unsigned char*>(scratch);
  auto* counter = reinterpret_cast<uint32_t*>(base);
  auto* part_v = reinterpret_cast<float*>(base + 16);
  auto* part_i = reinterpret_cast<int32_t*>(base + 16 + 4 * kArgMaxCtas);
  static_assert(16 + 8 * kArgMaxCtas <= kArgmaxScratchBytes, "argmax scratch");
  return launch_pdl(k_argmax, dim3(ctas), dim3(kArgThreads), st, logits, n, per_cta, token, value, part_v, part_i,
                    counter);
}

}  // namespace b2a
