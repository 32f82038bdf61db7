// Projections with int8 weights, one scale per output row (the reference's
// symmetric per-channel scheme, src/core/quantize.js:36-58), for the layers
// either side of attention: out[t][r] = res[t][r] + scale[r] * sum_c W[r][c] x[t][c]
// + bias[r] (matVec, src/core/ops.js:33-41, applied per token; o_proj's
// residual add, src/cpu/model.js:125-128).
//
// Tensor cores (mma.sync m16n8k16, f16 in, f32 accumulate): an int8 code is
// exact in f16, so A = the codes of 16 rows and the row scale is applied in the
// epilogue; B = the activations, split into an f16 high part and an f16
// residual (two MMAs) so the product keeps ~f32 precision. A CTA of eight warps
// owns 16 rows x 32 tokens (so a 1152-row projection spreads over 72 CTAs even
// for one token) and stages its weight rows (int8) and the tokens' activations
// (as given: f32, f16 or bf16) in shared memory for up to 1024 columns at a
// time with asynchronous 16-byte copies, all in flight at once. The eight warps
// split the columns, MMA only the 8-token tiles that hold tokens, and add their
// partial sums through shared memory. Weight reads dominate the bytes
// (HBM-bound for large matrices; latency-bound at the Qwen2.5-0.5B sizes).
#include <cuda_fp16.h>

#include "b2a_internal.cuh"
#include "k_util.cuh"

namespace b2a {

namespace {

constexpr int kRowsPerCta = 16;
constexpr int kTokPerCta = 32;
constexpr int kMaxKc = 1024;                    // columns staged per pass
constexpr int kWPitch = kMaxKc + 16;            // bytes per staged weight row (bank spread)
constexpr int kXPitch = kMaxKc * 4 + 16;        // bytes per staged token row (f32 or 16-bit)
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kSmem = kRowsPerCta * kWPitch + kTokPerCta * kXPitch + kWarps * kRowsPerCta * kTokPerCta * 4;

// 16-byte asynchronous copy global -> shared; src_bytes 0 fills zeros
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(src_bytes)
               : "memory");
}

// two int8 codes (low byte first) -> f16x2, exactly: 1024 + (q + 128) is an
// f16 with the byte in its low mantissa bits, minus 1152
__device__ __forceinline__ uint32_t i8x2_to_h2(uint32_t v16) {
  const uint32_t t = __byte_perm(v16 ^ 0x8080u, 0x6464u, 0x5140);
  __half2 h = *reinterpret_cast<const __half2*>(&t);
  h = __hsub2(h, __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));   // 1152
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

}  // namespace

__global__ void __launch_bounds__(kThreads) k_linear_int8(LinearParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* ws = smem;                                                 // [16][kWPitch] int8 codes
  unsigned char* xs = smem + kRowsPerCta * kWPitch;                         // [32][kXPitch] activations as given
  float* part = reinterpret_cast<float*>(xs + kTokPerCta * kXPitch);       // [8 warps][16 rows][32 tokens]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int r0 = blockIdx.x * kRowsPerCta;
  const int t0 = blockIdx.y * kTokPerCta;
  const int nrows = min(kRowsPerCta, p.rows - r0);
  const int ntok = min(kTokPerCta, p.tokens - t0);
  const int ntiles = (ntok + 7) / 8;             // 8-token MMA tiles that hold tokens
  const int esz = p.x_dtype == DT_F32 ? 4 : 2;

  // Programmatic dependent launch: the next kernel may start its prologue
  // once every CTA of this grid is resident; this grid reads nothing from
  // global memory before the kernel ahead of it (which may have written the
  // weights, scales or activations) has finished.
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // the rows' scales and biases, loaded while the tiles stream in
  __shared__ float rsc[kRowsPerCta], rbi[kRowsPerCta];
  if (tid < kRowsPerCta) {
    const int r = r0 + tid;
    rsc[tid] = tid < nrows ? ld_as_f32(p.scale, r, p.scale_dtype) : 0.f;
    rbi[tid] = (tid < nrows && p.bias) ? ld_as_f32(p.bias, r, p.bias_dtype) : 0.f;
  }

  float acc[4][4];
#pragma unroll
  for (int n = 0; n < 4; n++)
#pragma unroll
    for (int e = 0; e < 4; e++) acc[n][e] = 0.f;

  for (int c0 = 0; c0 < p.cols; c0 += kMaxKc) {
    const int kc = min(kMaxKc, p.cols - c0);   // a multiple of 16
    if (c0 > 0) __syncthreads();                 // the previous pass is done with the tiles
    const int wvec = kc / 16;
    for (int i = tid; i < kRowsPerCta * wvec; i += kThreads) {
      const int r = i / wvec, v = i % wvec;
      const bool in = r < nrows;
      cp_async16(ws + r * kWPitch + 16 * v, p.w + (in ? static_cast<int64_t>(r0 + r) * p.cols + c0 + 16 * v : 0),
                 in ? 16 : 0);
    }
    // only the tokens that exist (the rest of a tile reads stale shared
    // memory, which only reaches that tile's unused output columns)
    const int xvec = kc * esz / 16;
    for (int i = tid; i < ntok * xvec; i += kThreads) {
      const int t = i / xvec, v = i % xvec;
      cp_async16(xs + t * kXPitch + 16 * v,
                 static_cast<const unsigned char*>(p.x) + (static_cast<int64_t>(t0 + t) * p.cols + c0) * esz + 16 * v, 16);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const unsigned char* wr0 = ws + gq * kWPitch;
    const unsigned char* wr1 = wr0 + 8 * kWPitch;
    // this warp's eighth of the staged columns, in 16-column steps
    const int steps = kc / 16;
    const int k_begin = 16 * ((steps * warp) / kWarps), k_end = 16 * ((steps * (warp + 1)) / kWarps);
    for (int k = k_begin; k < k_end; k += 16) {
      const uint32_t a0 = i8x2_to_h2(*reinterpret_cast<const uint16_t*>(wr0 + k + 2 * tq));
      const uint32_t a1 = i8x2_to_h2(*reinterpret_cast<const uint16_t*>(wr1 + k + 2 * tq));
      const uint32_t a2 = i8x2_to_h2(*reinterpret_cast<const uint16_t*>(wr0 + k + 8 + 2 * tq));
      const uint32_t a3 = i8x2_to_h2(*reinterpret_cast<const uint16_t*>(wr1 + k + 8 + 2 * tq));
#pragma unroll
      for (int n = 0; n < 4; n++) {
        if (n >= ntiles) break;
        const unsigned char* xr = xs + (8 * n + gq) * kXPitch;
        float v[4];   // x[t][k+2tq], x[t][k+2tq+1], x[t][k+8+2tq], x[t][k+9+2tq]
        if (esz == 4) {
          const float2 f0 = *reinterpret_cast<const float2*>(xr + 4 * (k + 2 * tq));
          const float2 f1 = *reinterpret_cast<const float2*>(xr + 4 * (k + 8 + 2 * tq));
          v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
        } else {
          const uint32_t u0 = *reinterpret_cast<const uint32_t*>(xr + 2 * (k + 2 * tq));
          const uint32_t u1 = *reinterpret_cast<const uint32_t*>(xr + 2 * (k + 8 + 2 * tq));
          const int dt = p.x_dtype;
          v[0] = dt == DT_F16 ? __half2float(__ushort_as_half(u0 & 0xffff)) : __uint_as_float(u0 << 16);
          v[1] = dt == DT_F16 ? __half2float(__ushort_as_half(u0 >> 16)) : __uint_as_float(u0 & 0xffff0000u);
          v[2] = dt == DT_F16 ? __half2float(__ushort_as_half(u1 & 0xffff)) : __uint_as_float(u1 << 16);
          v[3] = dt == DT_F16 ? __half2float(__ushort_as_half(u1 >> 16)) : __uint_as_float(u1 & 0xffff0000u);
        }
        const __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
        const float2 g0 = __half22float2(h0), g1 = __half22float2(h1);
        const __half2 l0 = __floats2half2_rn(v[0] - g0.x, v[1] - g0.y), l1 = __floats2half2_rn(v[2] - g1.x, v[3] - g1.y);
        mma_f16(acc[n], a0, a1, a2, a3, *reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
        mma_f16(acc[n], a0, a1, a2, a3, *reinterpret_cast<const uint32_t*>(&l0), *reinterpret_cast<const uint32_t*>(&l1));
      }
    }
  }

  // the warps' partial sums: C fragment (rows gq / gq+8, tokens 2tq, 2tq+1 of
  // each tile) -> part[warp][row][token], then a thread per (row, token)
#pragma unroll
  for (int n = 0; n < 4; n++) {
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int row = gq + 8 * (e >> 1), tok = 8 * n + 2 * tq + (e & 1);
      part[(warp * kRowsPerCta + row) * kTokPerCta + tok] = acc[n][e];
    }
  }
  __syncthreads();
  // two (row, token) outputs per thread: every global load first, then the math
  constexpr int kPer = kRowsPerCta * kTokPerCta / kThreads;
  float res[kPer];
#pragma unroll
  for (int u = 0; u < kPer; u++) {
    const int i = tid + kThreads * u, row = i / kTokPerCta, tok = i % kTokPerCta;
    res[u] = 0.f;
    if (p.residual && row < nrows && tok < ntok) {
      const int r = r0 + row;
      const int seg_rows = p.seg_end[0];   // the residual comes with one segment
      res[u] = ld_as_f32(p.residual, static_cast<int64_t>(t0 + tok) * seg_rows + r, p.out_dtype);
    }
  }
#pragma unroll
  for (int u = 0; u < kPer; u++) {
    const int i = tid + kThreads * u, row = i / kTokPerCta, tok = i % kTokPerCta;
    const int r = r0 + row, t = t0 + tok;
    float sum = 0.f;
#pragma unroll
    for (int w8 = 0; w8 < kWarps; w8++) sum += part[(w8 * kRowsPerCta + row) * kTokPerCta + tok];
    if (row >= nrows || tok >= ntok) continue;
    // the output segment of row r (selects, not indexing, keep the parameters in registers)
    const int seg = (p.nseg > 1 && r >= p.seg_end[0]) + (p.nseg > 2 && r >= p.seg_end[1]);
    const int seg_begin = seg == 0 ? 0 : (seg == 1 ? p.seg_end[0] : p.seg_end[1]);
    const int seg_rows = (seg == 0 ? p.seg_end[0] : (seg == 1 ? p.seg_end[1] : p.seg_end[2])) - seg_begin;
    void* out = seg == 0 ? p.out[0] : (seg == 1 ? p.out[1] : p.out[2]);
    const int64_t o = static_cast<int64_t>(t) * seg_rows + (r - seg_begin);
    st_from_f32(out, o, p.out_dtype, fmaf(sum, rsc[row], rbi[row]) + res[u]);
  }
}

cudaError_t launch_linear_int8(const LinearParams& p, cudaStream_t st) {
  if (p.rows <= 0 || p.tokens <= 0) return cudaSuccess;
  if (p.cols <= 0 || p.cols % 16 != 0 || p.nseg < 1 || p.nseg > 3) return cudaErrorInvalidValue;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr[64] = {};
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(k_linear_int8, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    attr[dev] = true;
  }
  const dim3 grid((p.rows + kRowsPerCta - 1) / kRowsPerCta, (p.tokens + kTokPerCta - 1) / kTokPerCta);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_linear_int8, p);
}

}  // namespace b2a
