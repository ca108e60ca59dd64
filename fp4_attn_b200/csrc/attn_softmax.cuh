// attn_softmax.cuh -- per-thread softmax and P requantization arithmetic of
// the attention kernel (one TMEM lane = one query row, 32 key columns per
// call), kept apart from the kernel's pipeline so it can be exercised alone.
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"

namespace fp4 {

// Shared-memory loads at 32-bit shared-window addresses.  The kernels re-align
// their dynamic shared memory base through an integer, after which the
// compiler cannot prove a pointer is shared and would issue generic loads
// (longer latency); volatile keeps them after the mbarrier waits that order
// them behind the asynchronous copies that filled the buffers.
__device__ __forceinline__ float4 lds_f4(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds_u2(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ float lds_f(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Packed fp32 pairs (sm_100a f32x2 ALU ops, each lane rounded like the scalar op).
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// E2M1 round-to-nearest-even of (x0, x1) (satfinite: |x| > 6 -> 6) -> the two
// fp16 values code * scale, with s14 = the block scale * 2^14 as two halves.
// The code byte is widened without the conversion pipe: for a 3-bit magnitude
// c, the fp16 bit pattern c << 9 is c's E2M1 value * 2^-14 (c = 1 lands on the
// fp16 subnormal 2^-15, c >= 2 on normals), so one multiply places both codes
// (low nibble -> bits 9..11, high nibble -> bits 25..27) and one mask cleans
// them.  P is non-negative, so the sign bits are dropped.  The products are
// exact in fp16: P's block scales lie in [2^-9, 0.171875] or are 0.
__device__ __forceinline__ uint32_t quant_pair_f16(float x0, float x1, uint32_t s14) {
  uint32_t c;
  asm("{\n\t.reg .b8 t;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n\t"
      "cvt.u32.u8 %0, t;\n\t}"
      : "=r"(c)
      : "f"(x0), "f"(x1));
  return hmul2_u32((c * 0x00200200u) & 0x0E000E00u, s14);
}

// Pass 1 on one 32-key chunk: running max of z = acc * gk (keys with
// column > lim masked when MASK); gk is the shared address of the chunk's 32
// key scales.  The products round like the packed ones of chunk_p.
template <bool MASK>
__device__ __forceinline__ float chunk_max(const uint32_t (&a)[32], uint32_t gk, int col0, int lim, float m) {
  float z[32];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 g = lds_f4(gk + 16 * q);
    z[4 * q] = __fmul_rn(__uint_as_float(a[4 * q]), g.x);
    z[4 * q + 1] = __fmul_rn(__uint_as_float(a[4 * q + 1]), g.y);
    z[4 * q + 2] = __fmul_rn(__uint_as_float(a[4 * q + 2]), g.z);
    z[4 * q + 3] = __fmul_rn(__uint_as_float(a[4 * q + 3]), g.w);
  }
  if constexpr (MASK) {
#pragma unroll
    for (int i = 0; i < 32; ++i) z[i] = (col0 + i > lim) ? -INFINITY : z[i];
  }
  // a tree (depth 4) instead of a chain of 16 dependent maxima
  float t[11];
#pragma unroll
  for (int i = 0; i < 10; ++i) t[i] = max3f(z[3 * i], z[3 * i + 1], z[3 * i + 2]);
  t[10] = fmaxf(z[30], z[31]);
  const float b0 = max3f(t[0], t[1], t[2]), b1 = max3f(t[3], t[4], t[5]), b2 = max3f(t[6], t[7], t[8]);
  const float b3 = max3f(t[9], t[10], m);
  return fmaxf(max3f(b0, b1, b2), b3);
}

// exp2 of four scores: e = exp2(acc * gk * u - m * u).
__device__ __forceinline__ void exp4(const uint32_t* a, float4 g, uint64_t u2, uint64_t nmu2, float* e) {
  float t0, t1, t2, t3;
  upk2(fma2(mul2(pk2(__uint_as_float(a[0]), __uint_as_float(a[1])), pk2(g.x, g.y)), u2, nmu2), t0, t1);
  upk2(fma2(mul2(pk2(__uint_as_float(a[2]), __uint_as_float(a[3])), pk2(g.z, g.w)), u2, nmu2), t2, t3);
  e[0] = ex2(t0);
  e[1] = ex2(t1);
  e[2] = ex2(t2);
  e[3] = ex2(t3);
}

// Block scale of 16 values of e: the E4M3 scale byte's reciprocal (rs) and
// the scale * 2^14 as two fp16 halves (s14).
__device__ __forceinline__ void block_scale(const float* eb, uint32_t rcp, float r6, uint64_t& rs2,
                                            uint32_t& s14) {
  const float m0 = max3f(eb[0], eb[1], eb[2]), m1 = max3f(eb[3], eb[4], eb[5]);
  const float m2 = max3f(eb[6], eb[7], eb[8]), m3 = max3f(eb[9], eb[10], eb[11]);
  const float m4 = max3f(eb[12], eb[13], eb[14]);
  const float amax = fmaxf(max3f(m0, m1, m2), max3f(m3, m4, eb[15]));
  const uint8_t sb = e4m3_satfinite(amax * r6);
  const float rs = lds_f(rcp + 4 * (sb & 127));
  rs2 = pk2(rs, rs);
  s14 = (uint32_t)__half_as_ushort(__float2half_rn(e4m3_to_f32(sb) * 16384.0f)) * 0x10001u;
}

// E2M1 round-to-nearest-even of (x0, x1) (satfinite), times the block scale:
// the fp16 pair code * s, exact (P's block scales lie in [2^-9, 0.171875] or are 0).
__device__ __forceinline__ uint32_t quant_pair_cvt(float x0, float x1, uint32_t s2) {
  uint32_t c;
  asm("{\n\t.reg .b8 t;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
      : "=r"(c)
      : "f"(x0), "f"(x1));
  return hmul2_u32(c, s2);
}

// The E4M3 scale byte b as an fp16 pair (exact: E4M3 values are fp16 values).
__device__ __forceinline__ uint32_t e4m3_f16x2(uint32_t b) {
  uint32_t r;
  asm("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(r) : "r"(b * 0x101u));
  return r;
}

// Block scale of 16 values of e without a table lookup (shared-memory loads
// wait behind the tensor core's operand reads while MMAs run): the scale as an
// fp16 pair (s2, exact) and 1/s by the hardware reciprocal (rs2; 0 for a zero
// block, as get_reciprocal gives).  1/s is within an ulp or two of the
// correctly rounded reciprocal the reference multiplies by, which moves only
// E2M1 decisions lying within ~1e-7 of a rounding boundary.
__device__ __forceinline__ void block_scale_rcp(const float* eb, float r6, uint64_t& rs2, uint32_t& s2) {
  const float m0 = max3f(eb[0], eb[1], eb[2]), m1 = max3f(eb[3], eb[4], eb[5]);
  const float m2 = max3f(eb[6], eb[7], eb[8]), m3 = max3f(eb[9], eb[10], eb[11]);
  const float m4 = max3f(eb[12], eb[13], eb[14]);
  const float amax = fmaxf(max3f(m0, m1, m2), max3f(m3, m4, eb[15]));
  s2 = e4m3_f16x2(e4m3_satfinite(amax * r6) & 127);
  const float sv = __half2float(__ushort_as_half((unsigned short)(s2 & 0xFFFFu)));
  float rs;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(rs) : "f"(sv));
  rs = sv == 0.0f ? 0.0f : rs;
  rs2 = pk2(rs, rs);
}

// Pass 2 on one 32-key chunk: e = exp2(z*u - m*u), running sum, NVFP4
// fake-quant of e in two blocks of 16 -> 16 words of fp16 pairs.  The exp2 of
// the second block is interleaved with the quantization of the first, so the
// MUFU and the conversion pipe work at the same time.
template <bool MASK>
__device__ __forceinline__ void chunk_p(const uint32_t (&a)[32], uint32_t gk, int col0, int lim, uint64_t u2,
                                        uint64_t nmu2, float r6, uint64_t (&lsum2)[4], uint32_t (&pk)[16]) {
  float e[32];
#pragma unroll
  for (int q = 0; q < 4; ++q) exp4(a + 4 * q, lds_f4(gk + 16 * q), u2, nmu2, e + 4 * q);
  if constexpr (MASK) {
#pragma unroll
    for (int i = 0; i < 16; ++i) e[i] = (col0 + i > lim) ? 0.0f : e[i];
  }
  uint64_t rs2;
  uint32_t s2;
  block_scale_rcp(e, r6, rs2, s2);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    exp4(a + 16 + 4 * q, lds_f4(gk + 64 + 16 * q), u2, nmu2, e + 16 + 4 * q);
#pragma unroll
    for (int i = 4 * q; i < 4 * q + 4; i += 2) {
      float x0, x1;
      upk2(mul2(pk2(e[i], e[i + 1]), rs2), x0, x1);
      pk[i / 2] = quant_pair_cvt(x0, x1, s2);
    }
  }
  if constexpr (MASK) {
#pragma unroll
    for (int i = 16; i < 32; ++i) e[i] = (col0 + i > lim) ? 0.0f : e[i];
  }
  block_scale_rcp(e + 16, r6, rs2, s2);
#pragma unroll
  for (int i = 16; i < 32; i += 2) {
    float x0, x1;
    upk2(mul2(pk2(e[i], e[i + 1]), rs2), x0, x1);
    pk[i / 2] = quant_pair_cvt(x0, x1, s2);
  }
#pragma unroll
  for (int i = 0; i < 32; i += 2) lsum2[(i >> 1) & 3] = add2(lsum2[(i >> 1) & 3], pk2(e[i], e[i + 1]));
}

// ---------------------------------------------------------------- dual-slice P
// The reference's dual_nvfp4 on P (fp4_quant_utils.py:307-315 via
// llama_patch.py:84-95): hi = qdq(P), lo = qdq(P - hi), both row-aligned
// (global scale = the row's max |.|), P-hat = hi + lo.  In the kernel's units
// (e = P / rowmax P) hi is the single-slice code * scale; the residual's row
// global scale gr = rowmax |e - hi| comes from an extra pass (chunk_rmax), and
// lo = (E2M1(x * rcp(s')) * s') * gr with x = (e - hi) * recip(gr) and
// s' = E4M3(max_block |x| * recip(6)), as fp4_quant_utils.py:118-169 does.

// e = exp2(z*u - m*u) of one 32-key chunk (keys with column > lim zeroed when MASK).
template <bool MASK>
__device__ __forceinline__ void chunk_e(const uint32_t (&a)[32], uint32_t gk, int col0, int lim, uint64_t u2,
                                        uint64_t nmu2, float (&e)[32]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) exp4(a + 4 * q, lds_f4(gk + 16 * q), u2, nmu2, e + 4 * q);
  if constexpr (MASK) {
#pragma unroll
    for (int i = 0; i < 32; ++i) e[i] = (col0 + i > lim) ? 0.0f : e[i];
  }
}

// hi slice of 16 values: fp16 pairs code * scale (exact), as chunk_p forms them.
__device__ __forceinline__ void slice_hi(const float* eb, uint32_t rcp, float r6, uint32_t (&hp)[8]) {
  uint64_t rs2;
  uint32_t s14;
  block_scale(eb, rcp, r6, rs2, s14);
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    float x0, x1;
    upk2(mul2(pk2(eb[i], eb[i + 1]), rs2), x0, x1);
    hp[i / 2] = quant_pair_f16(x0, x1, s14);
  }
}

__device__ __forceinline__ float2 f16x2_to_f32(uint32_t h) {
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// Residual pass on one 32-key chunk: running max of |e - hi|.
template <bool MASK>
__device__ __forceinline__ float chunk_rmax(const uint32_t (&a)[32], uint32_t gk, int col0, int lim, uint64_t u2,
                                            uint64_t nmu2, uint32_t rcp, float r6, float rm) {
  float e[32];
  chunk_e<MASK>(a, gk, col0, lim, u2, nmu2, e);
#pragma unroll
  for (int blk = 0; blk < 2; ++blk) {
    uint32_t hp[8];
    slice_hi(e + 16 * blk, rcp, r6, hp);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 h = f16x2_to_f32(hp[i]);
      rm = max3f(rm, fabsf(e[16 * blk + 2 * i] - h.x), fabsf(e[16 * blk + 2 * i + 1] - h.y));
    }
  }
  return rm;
}

// Final pass of dual-slice P on one 32-key chunk: running sum of e, then
// P-hat = hi + lo per key, rounded to fp16 pairs (pk).  rg = recip(gr).
template <bool MASK>
__device__ __forceinline__ void chunk_p_dual(const uint32_t (&a)[32], uint32_t gk, int col0, int lim, uint64_t u2,
                                             uint64_t nmu2, uint32_t rcp, float r6, float rg, float gr,
                                             uint64_t (&lsum2)[4], uint32_t (&pk)[16]) {
  float e[32];
  chunk_e<MASK>(a, gk, col0, lim, u2, nmu2, e);
#pragma unroll
  for (int i = 0; i < 32; i += 2) lsum2[(i >> 1) & 3] = add2(lsum2[(i >> 1) & 3], pk2(e[i], e[i + 1]));
  const uint64_t rg2 = pk2(rg, rg), gr2 = pk2(gr, gr);
#pragma unroll
  for (int blk = 0; blk < 2; ++blk) {
    const float* eb = e + 16 * blk;
    uint32_t hp[8];
    slice_hi(eb, rcp, r6, hp);
    float xr[16];
    float am = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 h = f16x2_to_f32(hp[i]);
      upk2(mul2(add2(pk2(eb[2 * i], eb[2 * i + 1]), pk2(-h.x, -h.y)), rg2), xr[2 * i], xr[2 * i + 1]);
      am = max3f(am, fabsf(xr[2 * i]), fabsf(xr[2 * i + 1]));
    }
    const uint32_t sb = e4m3_satfinite(am * r6);
    const float rs = lds_f(rcp + 4 * (sb & 127));
    const uint64_t rs2 = pk2(rs, rs);
    uint32_t s2;
    asm("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(s2) : "r"(sb * 0x101u));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float x0, x1;
      upk2(mul2(pk2(xr[2 * i], xr[2 * i + 1]), rs2), x0, x1);
      uint32_t qs;  // (E2M1(x) * s') as fp16 pair, exact, signed
      asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n\t"
          "cvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
          : "=r"(qs)
          : "f"(x0), "f"(x1));
      qs = hmul2_u32(qs, s2);
      const float2 lq = f16x2_to_f32(qs);
      const float2 h = f16x2_to_f32(hp[i]);
      float p0, p1;
      upk2(add2(pk2(h.x, h.y), mul2(pk2(lq.x, lq.y), gr2)), p0, p1);
      uint32_t w;
      asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(w) : "f"(p1), "f"(p0));
      pk[8 * blk + i] = w;
    }
  }
}

}  // namespace fp4
