// Device helpers: dtype conversion with the reference's rounding rules, and the
// f64 RoPE rotation.
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>

namespace b2a {

enum { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };

__device__ __forceinline__ float ld_as_f32(const void* base, int64_t i, int dt) {
  if (dt == DT_F32) return static_cast<const float*>(base)[i];
  if (dt == DT_F16) return __half2float(static_cast<const __half*>(base)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
}

// f32 -> f16 bits, round to nearest even (src/core/dtype.js:81-113). The
// hardware conversion is RNE with overflow to inf and gradual underflow; only
// NaN differs (hardware canonicalises), so NaN takes the reference's rule:
// keep the sign, force a quiet payload bit.
__device__ __forceinline__ uint16_t f32_to_f16_bits(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu) != 0u) {
    uint32_t sign = (u >> 16) & 0x8000u;
    return static_cast<uint16_t>(sign | 0x7c00u | ((u & 0x7fffffu) >> 13) | 0x200u);
  }
  return __half_as_ushort(__float2half_rn(x));
}

// f32 -> bf16 bits, round to nearest even (src/core/dtype.js:23-35).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu) != 0u) {
    return static_cast<uint16_t>(((u >> 16) | 0x0040u) & 0xffffu);
  }
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

__device__ __forceinline__ void st_from_f32(void* base, int64_t i, int dt, float x) {
  if (dt == DT_F32) {
    static_cast<float*>(base)[i] = x;
  } else if (dt == DT_F16) {
    static_cast<uint16_t*>(base)[i] = f32_to_f16_bits(x);
  } else {
    static_cast<uint16_t*>(base)[i] = f32_to_bf16_bits(x);
  }
}

// Copy one element between dtypes with the reference's rounding: a value that
// already has the destination dtype is copied bit for bit.
__device__ __forceinline__ void convert_elem(const void* src, int64_t si, int sdt, void* dst, int64_t di, int ddt) {
  if (sdt == ddt) {
    if (sdt == DT_F32) static_cast<uint32_t*>(dst)[di] = static_cast<const uint32_t*>(src)[si];
    else static_cast<uint16_t*>(dst)[di] = static_cast<const uint16_t*>(src)[si];
    return;
  }
  st_from_f32(dst, di, ddt, ld_as_f32(src, si, sdt));
}

// src/core/ops.js:153-156 in IEEE f64 with every product and sum rounded
// separately (no FMA contraction, as JavaScript evaluates it), stored to f32.
__device__ __forceinline__ void rope_pair_f64(float lo, float hi, double c, double s, float& out_lo,
                                              float& out_hi) {
  double dlo = static_cast<double>(lo), dhi = static_cast<double>(hi);
  out_lo = __double2float_rn(__dsub_rn(__dmul_rn(dlo, c), __dmul_rn(dhi, s)));
  out_hi = __double2float_rn(__dadd_rn(__dmul_rn(dhi, c), __dmul_rn(dlo, s)));
}

}  // namespace b2a
