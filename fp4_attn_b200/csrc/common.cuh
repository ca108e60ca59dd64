// common.cuh -- device helpers shared by the NVFP4 kernels (sm_100a).
//
// Arithmetic conventions (the reference's torch path, fp4_quant_utils.py):
//  * every elementwise op of the reference computes in fp32 and rounds once
//    to the dequant dtype; rnd<A>() is that rounding;
//  * products use __fmul_rn and reciprocals __frcp_rn so nvcc never fuses or
//    approximates them (the build also passes --fmad=false);
//  * NaN propagates through max (torch.max/amax), so maxima use max.NaN.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define FP4_ARITH_F32 0
#define FP4_ARITH_BF16 1
#define FP4_ARITH_F16 2

#define FP4_DT_F32 0
#define FP4_DT_BF16 1
#define FP4_DT_F16 2

namespace fp4 {

template <int A>
__device__ __forceinline__ float rnd(float v) {
  if constexpr (A == FP4_ARITH_BF16) {
    return __bfloat162float(__float2bfloat16_rn(v));
  } else if constexpr (A == FP4_ARITH_F16) {
    return __half2float(__float2half_rn(v));
  } else {
    return v;
  }
}

// a*b in the dequant dtype.
template <int A>
__device__ __forceinline__ float mul(float a, float b) {
  return rnd<A>(__fmul_rn(a, b));
}

// get_reciprocal (fp4_quant_utils.py:64-69): 0 where v == 0, else 1/v.
template <int A>
__device__ __forceinline__ float recip(float v) {
  return v == 0.0f ? 0.0f : rnd<A>(__frcp_rn(v));
}

// recip<A>(6.0f) as a compile-time constant: 1.0f / 6.0f is folded with IEEE
// round-to-nearest, the rounding rcp.rn gives, so no reciprocal runs per block.
template <int A>
__device__ __forceinline__ float recip6() {
  constexpr float kSixth = 1.0f / 6.0f;
  return rnd<A>(kSixth);
}

// NaN-propagating maximum (torch.max semantics).
__device__ __forceinline__ float nanmax(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// max(|a|,|b|,|c|) with NaN winning.
__device__ __forceinline__ float absmax3(float a, float b, float c) {
  float r;
  asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// torch's float32 -> float8_e4m3fn cast: round to nearest even, any
// magnitude above 464 (and NaN) becomes NaN (0x7F with the sign bit).
__device__ __forceinline__ uint8_t e4m3_torch(float v) {
  uint8_t b = (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
  if (!(fabsf(v) <= 464.0f)) b = (uint8_t)((__float_as_uint(v) >> 24) & 0x80u) | 0x7Fu;
  return b;
}

// __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3): saturates to 448.
__device__ __forceinline__ uint8_t e4m3_satfinite(float v) {
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
  return __half2float(__half(__nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3)));
}

// Two floats -> one byte of E2M1 codes (a in the low nibble), round to
// nearest even, saturating at +-6.  The sign of zero is kept: callers that
// need torch.sign's +0 for -0.0 add +0.0 first.
__device__ __forceinline__ uint32_t e2m1x2(float a, float b) {
  uint16_t r;
  asm("{\n\t.reg .b8 t;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n\t"
      "cvt.u16.u8 %0, t;\n\t}"
      : "=h"(r)
      : "f"(a), "f"(b));
  return r;
}

// Value of an E2M1 code nibble.
__device__ __forceinline__ float e2m1_value(uint32_t c) {
  const float mag = (c & 4) ? ((c & 2) ? ((c & 1) ? 6.0f : 4.0f) : ((c & 1) ? 3.0f : 2.0f))
                            : ((c & 2) ? ((c & 1) ? 1.5f : 1.0f) : ((c & 1) ? 0.5f : 0.0f));
  return (c & 8) ? -mag : mag;
}

template <int DT>
struct In;
template <>
struct In<FP4_DT_F32> {
  using T = float;
  static __device__ __forceinline__ float f(float v) { return v; }
};
template <>
struct In<FP4_DT_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float f(__nv_bfloat16 v) { return __bfloat162float(v); }
};
template <>
struct In<FP4_DT_F16> {
  using T = __half;
  static __device__ __forceinline__ float f(__half v) { return __half2float(v); }
};

template <int DT>
__device__ __forceinline__ void store_out(void* p, int64_t i, float v) {
  if constexpr (DT == FP4_DT_BF16) {
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  } else if constexpr (DT == FP4_DT_F16) {
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  } else {
    reinterpret_cast<float*>(p)[i] = v;
  }
}

// Byte offset of block-scale (row r, 16-element block kb) in the tcgen05
// block-scaled MMA layout: 128-row x 4-block atoms of 512 bytes, atoms
// ordered k-fastest; inside an atom, row r sits at (r%32)*16 + ((r/32)%4)*4
// and block kb at kb%4.  nkb4 = number of 4-block groups per row.
__device__ __host__ __forceinline__ int64_t sf_tcgen05_offset(int64_t r, int64_t kb, int64_t nkb4) {
  return ((r >> 7) * nkb4 + (kb >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (kb & 3);
}

}  // namespace fp4
