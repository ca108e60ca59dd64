// quant_impl.cuh -- NVFP4 quantize / fused quantize-dequantize kernels (sm_100a).
// Included once per input dtype by quant_{f32,bf16,f16}.cu so the template
// fan-out compiles in parallel; quant.cu holds the C ABI entry points.
//
// Bit-exact restatement of FP4Quantizer.single_nvfp4_quant_dequant_fused
// (fp4_quant_utils.py:112-172) that also emits what the reference only
// implies: packed E2M1 codes, E4M3 block-scale bytes and the global scales.
//
// Layout.  The input is a logical matrix whose row is (b, t) and whose
// column is c = h*D + d, element at x[b*sB + t*sT + h*sH + d] (d contiguous).
// A plain 2-D [m, n] tensor is B=1, T=m, H=1, D=n.  The [B,H,T,D] attention
// operands of llama_patch.py:167-169 ([B*T, H*D] views) use the same kernel
// without a transpose copy.  Output row index is b*T_pad + t; rows t >= T
// are padding and are written as zeros (codes, scales and g).
//
// Work split.  A CTA has 128 threads; TPR threads own one row (TPR = 32, 64
// or 128) and each thread owns 16-element blocks kb = lane + i*TPR, loaded
// with 16-byte vector loads when the row is aligned.  Row mode needs the
// row's |x| maximum before any block is quantized: up to MAXB blocks per
// thread stay in registers between the two phases, longer rows are re-read
// (from L1/L2).  Column and tensor modes take their global scale from a
// pre-pass (colmax / absmax kernels, atomicMax on the bits of |x|, which
// orders non-negative floats and lets NaN win, as torch.max does).
#pragma once
#include <stdio.h>

#include <algorithm>

#include "common.cuh"
#include "status.h"

namespace fp4 {

constexpr int kThreads = 128;
constexpr int kVecThreads = 256;  // quant_rows_vec_kernel
constexpr int MAXB = 2;  // 16-element blocks a thread keeps in registers

struct QuantArgs {
  const void* x;
  int64_t sB, sT, sH;
  int B, T, H, D;
  int T_pad;
  int vec;  // 16-byte aligned rows: vector loads
  int gmode;
  const float* g_in;  // col: [npad] final g; tensor: [1] final g
  float* g_row;       // row mode: [B*T_pad] (nullable)
  uint8_t* codes;
  int64_t codes_ld;  // bytes per output row
  uint8_t* scales;
  int scale_layout;  // 0 linear, 1 tcgen05 atoms
  int64_t scales_ld;  // linear: bytes per row; tcgen05: 4-block groups per row
  void* out;
  int64_t out_ld;  // elements per output row
  // dual-slice row mode (quant_rows_vec_kernel<..., DUAL>): the second slice's
  // codes / scales (same layouts as codes / scales) and per-row g
  uint8_t* codes_lo;
  uint8_t* scales_lo;
  float* g_row_lo;
};

template <int DT, int A>
__device__ __forceinline__ void load_block(float v[16], const QuantArgs& p, int b, int t, int kb) {
  using T = typename In<DT>::T;
  const int64_t n = (int64_t)p.H * p.D;
  const int64_t c0 = (int64_t)kb * 16;
  const T* base = reinterpret_cast<const T*>(p.x) + (int64_t)b * p.sB + (int64_t)t * p.sT;
  if (p.vec && c0 + 16 <= n) {
    const int h = (int)c0 / p.D;
    const int d = (int)c0 - h * p.D;
    const T* q = base + (int64_t)h * p.sH + d;
    if constexpr (DT == FP4_DT_F32) {
      const float4* q4 = reinterpret_cast<const float4*>(q);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float4 f = __ldg(q4 + j);
        v[4 * j + 0] = rnd<A>(f.x);
        v[4 * j + 1] = rnd<A>(f.y);
        v[4 * j + 2] = rnd<A>(f.z);
        v[4 * j + 3] = rnd<A>(f.w);
      }
    } else {
      const uint4* q4 = reinterpret_cast<const uint4*>(q);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint4 u = __ldg(q4 + j);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if constexpr (DT == FP4_DT_BF16) {
            v[8 * j + 2 * k] = rnd<A>(__uint_as_float(w[k] << 16));
            v[8 * j + 2 * k + 1] = rnd<A>(__uint_as_float(w[k] & 0xFFFF0000u));
          } else {
            const __half2 h2 = *reinterpret_cast<const __half2*>(&w[k]);
            const float2 f2 = __half22float2(h2);
            v[8 * j + 2 * k] = rnd<A>(f2.x);
            v[8 * j + 2 * k + 1] = rnd<A>(f2.y);
          }
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int64_t c = c0 + j;
      float f = 0.0f;
      if (c < n) {
        const int h = (int)(c / p.D);
        const int d = (int)(c - (int64_t)h * p.D);
        f = In<DT>::f(base[(int64_t)h * p.sH + d]);
      }
      v[j] = rnd<A>(f);
    }
  }
}

__device__ __forceinline__ float block_absmax(const float v[16]) {
  float m0 = absmax3(v[0], v[1], v[2]);
  float m1 = absmax3(v[3], v[4], v[5]);
  float m2 = absmax3(v[6], v[7], v[8]);
  float m3 = absmax3(v[9], v[10], v[11]);
  float m4 = absmax3(v[12], v[13], v[14]);
  m0 = absmax3(m0, m1, m2);
  m3 = absmax3(m3, m4, v[15]);
  return nanmax(m0, m3);
}

// Packed fp32 pair ops (sm_100a), exact IEEE round-to-nearest per lane.
__device__ __forceinline__ void mul2(float& a, float& b, float s) {
  uint64_t x, y;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a), "f"(b));
  asm("mov.b64 %0, {%1, %1};" : "=l"(y) : "f"(s));
  asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(x) : "l"(y));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(x));
}

// (a*s + 0, b*s + 0): one rounding of the product; the + 0 turns -0.0 into
// +0.0 like torch.sign(-0.0) == 0 does in cast_to_fp4 (fp4_quant_utils.py:49,62).
__device__ __forceinline__ void mulz2(float& a, float& b, float s) {
  uint64_t x, y, z = 0;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a), "f"(b));
  asm("mov.b64 %0, {%1, %1};" : "=l"(y) : "f"(s));
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(z) : "l"(x), "l"(y));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(z));
}

// Eight floats -> one word of E2M1 codes (element k in nibble k), RNE, satfinite.
__device__ __forceinline__ uint32_t e2m1x8(const float* v) {
  uint32_t r;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(r)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return r;
}

// Quantize one block of 16 (values already in the dequant dtype, before the
// global scale) and write its codes / scale byte / dequantized values.
// COLG: per-column global scale (column mode), else the scalar g / rg
// (row and tensor modes; none mode runs with g = rg = 1, which is exact).
template <int A, int ODT, bool COLG, bool OUT>
__device__ __forceinline__ void quant_block(float v[16], const QuantArgs& p, int64_t orow, int kb, float g, float rg,
                                            const float* rcp_tab, uint32_t* wout = nullptr, float* sout = nullptr) {
  const float r6 = recip6<A>();
  if constexpr (COLG) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = mul<A>(v[j], recip<A>(p.g_in[kb * 16 + j]));
  } else if constexpr (A == FP4_ARITH_F32) {
#pragma unroll
    for (int j = 0; j < 16; j += 2) mul2(v[j], v[j + 1], rg);
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = mul<A>(v[j], rg);
  }
  const float amax = block_absmax(v);
  const uint8_t sb = e4m3_torch(mul<A>(amax, r6));
  const float s = e4m3_to_f32(sb);
  const float rs = rcp_tab[sb & 0x7F];  // recip<A>(s); sb < 0x80 (amax >= 0)
  const bool nan_block = (sb & 0x7F) == 0x7F;
  if constexpr (A == FP4_ARITH_F32) {
#pragma unroll
    for (int j = 0; j < 16; j += 2) mulz2(v[j], v[j + 1], rs);
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = rnd<A>(__fmaf_rn(v[j], rs, 0.0f));
  }
  uint32_t w[2];
  w[0] = nan_block ? 0u : e2m1x8(v);
  w[1] = nan_block ? 0u : e2m1x8(v + 8);
  if (wout) {  // the block's codes and scale, for a caller that needs the dequantized values
    wout[0] = w[0];
    wout[1] = w[1];
    *sout = s;
  }
  if (p.codes) {
    *reinterpret_cast<uint2*>(p.codes + orow * p.codes_ld + (int64_t)kb * 8) = make_uint2(w[0], w[1]);
  }
  if (p.scales) {
    const int64_t off = p.scale_layout ? sf_tcgen05_offset(orow, kb, p.scales_ld) : orow * p.scales_ld + kb;
    p.scales[off] = sb;
  }
  if constexpr (OUT) {
    const int64_t n = (int64_t)p.H * p.D;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int64_t c = (int64_t)kb * 16 + j;
      if (c < n) {
        float o = mul<A>(e2m1_value((w[j >> 3] >> (4 * (j & 7))) & 15u), s);
        if constexpr (COLG) o = mul<A>(o, p.g_in[c]);
        else o = mul<A>(o, g);
        store_out<ODT>(p.out, orow * p.out_ld + c, o);
      }
    }
  }
}

template <int DT, int A, int ODT, int TPR, bool COLG, bool OUT>
__global__ void __launch_bounds__(kThreads, 8) quant_rows_kernel(QuantArgs p) {
  constexpr int ROWS = kThreads / TPR;
  constexpr int WPR = TPR / 32;  // warps per row
  __shared__ float red[kThreads / 32];
  __shared__ float rcp_tab[128];  // recip<A> of every non-negative E4M3 scale byte
  {
    const float sv = e4m3_to_f32((uint8_t)threadIdx.x);
    rcp_tab[threadIdx.x] = recip<A>(sv);
  }
  __syncthreads();
  const int rloc = threadIdx.x / TPR;
  const int lane = threadIdx.x % TPR;
  const int64_t orow = (int64_t)blockIdx.x * ROWS + rloc;
  const int64_t nrows = (int64_t)p.B * p.T_pad;
  const int64_t n = (int64_t)p.H * p.D;
  const int nblk = (int)((n + 15) / 16);
  const bool live = orow < nrows;
  const int b = live ? (int)(orow / p.T_pad) : 0;
  const int t = live ? (int)(orow - (int64_t)b * p.T_pad) : 0;
  const bool pad_row = !live || t >= p.T;
  const int nmine = lane < nblk ? (nblk - lane + TPR - 1) / TPR : 0;  // blocks this thread owns

  float cache[MAXB][16];
  // First chunk of this thread's blocks: all loads issued before any math.
  if (!pad_row) {
#pragma unroll
    for (int i = 0; i < MAXB; ++i)
      if (i < nmine) load_block<DT, A>(cache[i], p, b, t, lane + i * TPR);
  }
  float g = 1.0f;
  if (p.gmode == 1) {
    float m = 0.0f;
    if (!pad_row) {
#pragma unroll
      for (int i = 0; i < MAXB; ++i)
        if (i < nmine) m = nanmax(m, block_absmax(cache[i]));
      for (int i = MAXB; i < nmine; ++i) {
        float v[16];
        load_block<DT, A>(v, p, b, t, lane + i * TPR);
        m = nanmax(m, block_absmax(v));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = nanmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (WPR > 1) {
      if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = m;
      __syncthreads();
      m = red[rloc * WPR];
#pragma unroll
      for (int w = 1; w < WPR; ++w) m = nanmax(m, red[rloc * WPR + w]);
    }
    g = m;  // rowmax, no division by global_sf_max (fp4_quant_utils.py:134,139)
    if (p.g_row && lane == 0 && live) p.g_row[orow] = pad_row ? 0.0f : g;
  } else if (p.gmode == 3) {
    g = p.g_in[0];
  }
  if (!live) return;
  if (pad_row) {
    for (int kb = lane; kb < nblk; kb += TPR) {
      if (p.codes) *reinterpret_cast<uint2*>(p.codes + orow * p.codes_ld + (int64_t)kb * 8) = make_uint2(0u, 0u);
      if (p.scales) p.scales[p.scale_layout ? sf_tcgen05_offset(orow, kb, p.scales_ld) : orow * p.scales_ld + kb] = 0;
    }
    return;
  }
  const float rg = p.gmode == 0 ? 1.0f : recip<A>(g);
#pragma unroll
  for (int i = 0; i < MAXB; ++i)
    if (i < nmine) quant_block<A, ODT, COLG, OUT>(cache[i], p, orow, lane + i * TPR, g, rg, rcp_tab);
  for (int i = MAXB; i < nmine; ++i) {
    float v[16];
    load_block<DT, A>(v, p, b, t, lane + i * TPR);
    quant_block<A, ODT, COLG, OUT>(v, p, orow, lane + i * TPR, g, rg, rcp_tab);
  }
}

// Column / tensor maxima of |x| (in the dequant dtype) into bits[]:
// each thread owns 8 consecutive columns (one 16-byte load per row) of a
// slab of rows.
template <int DT, int A>
__global__ void __launch_bounds__(256) absmax_kernel(QuantArgs p, unsigned int* bits, int per_column) {
  using T = typename In<DT>::T;
  const int64_t n = (int64_t)p.H * p.D;
  const int64_t nrows = (int64_t)p.B * p.T;
  const int64_t c0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const int64_t rows_per = (nrows + gridDim.y - 1) / gridDim.y;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per;
  const int64_t r1 = r0 + rows_per < nrows ? r0 + rows_per : nrows;
  float m[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) m[j] = 0.0f;
  const bool vec = p.vec && c0 + 8 <= n && (p.H == 1 || (c0 % p.D) + 8 <= p.D) && (sizeof(T) == 2);
  for (int64_t r = r0; r < r1; ++r) {
    const int b = (int)r / p.T;
    const int t = (int)r - b * p.T;
    const T* row = reinterpret_cast<const T*>(p.x) + (int64_t)b * p.sB + (int64_t)t * p.sT;
    if (vec) {
      const int h = (int)c0 / p.D;
      const int d = (int)c0 - h * p.D;
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(row + (int64_t)h * p.sH + d));
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) m[j] = nanmax(m[j], fabsf(rnd<A>(In<DT>::f(e[j]))));
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t c = c0 + j;
        if (c < n) {
          const int h = (int)(c / p.D);
          const int d = (int)(c - (int64_t)h * p.D);
          m[j] = nanmax(m[j], fabsf(rnd<A>(In<DT>::f(row[(int64_t)h * p.sH + d]))));
        }
      }
    }
  }
  if (per_column) {
    if (r1 > r0) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (c0 + j < n) atomicMax(bits + c0 + j, __float_as_uint(m[j]));
    }
    return;
  }
  float mm = m[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) mm = nanmax(mm, m[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mm = nanmax(mm, __shfl_xor_sync(0xffffffffu, mm, o));
  __shared__ float wmax[8];
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = mm;
  __syncthreads();
  if (threadIdx.x == 0) {
#pragma unroll
    for (int w = 1; w < 8; ++w) mm = nanmax(mm, wmax[w]);
    atomicMax(bits, __float_as_uint(mm));
  }
}

// Tensor maximum of |x| for a contiguous input (the whole tensor is one run
// of nelem elements starting 16-byte aligned): grid-stride over 16-byte
// chunks, eight independent loads in flight per thread, one atomicMax per block
// (256 threads).
template <int DT, int A>
__global__ void __launch_bounds__(256) absmax_flat_kernel(const void* x, int64_t nelem, unsigned int* bits) {
  using T = typename In<DT>::T;
  constexpr int PER = 16 / sizeof(T);  // elements per 16-byte chunk
  const int64_t nchunk = nelem / PER;
  const uint4* src = reinterpret_cast<const uint4*>(x);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  float m = 0.0f;
  auto fold = [&](const uint4& u) {
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < PER; ++j) m = nanmax(m, fabsf(rnd<A>(In<DT>::f(e[j]))));
  };
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nchunk; i += 8 * stride) {
    uint4 u[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) u[k] = i + k * stride < nchunk ? __ldg(src + i + k * stride) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int k = 0; k < 8; ++k) fold(u[k]);
  }
  // the ragged tail (fewer than PER elements) goes to the first thread
  if (blockIdx.x == 0 && threadIdx.x == 0)
    for (int64_t k = nchunk * PER; k < nelem; ++k)
      m = nanmax(m, fabsf(rnd<A>(In<DT>::f(reinterpret_cast<const T*>(x)[k]))));
  // one atomic per block: same-address atomics serialise in L2
  __shared__ float wmax[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = nanmax(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
#pragma unroll
    for (int w = 1; w < 8; ++w) m = nanmax(m, wmax[w]);
    atomicMax(bits, __float_as_uint(m));
  }
}

// g = max * recip(global_sf_max) in the dequant dtype (fp4_quant_utils.py:139).
template <int A>
__global__ void finalize_g_kernel(float* g, int64_t count, float gsf_max) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) g[i] = mul<A>(g[i], recip<A>(rnd<A>(gsf_max)));
}

// Raw 16-byte vectors of one 16-element block (2 for 16-bit inputs, 4 for fp32).
template <int DT>
struct RawBlock {
  static constexpr int NV = DT == FP4_DT_F32 ? 4 : 2;
  uint4 u[NV];
};

// Element offset of block kb within a row: h * sH + d for c0 = 16 kb.
__device__ __forceinline__ int64_t block_col_offset(const QuantArgs& p, int kb) {
  const int c0 = kb * 16;
  const int h = c0 / p.D;
  return (int64_t)h * p.sH + (c0 - h * p.D);
}

template <int DT>
__device__ __forceinline__ void load_raw(RawBlock<DT>& r, const QuantArgs& p, int b, int t, int64_t col) {
  using T = typename In<DT>::T;
  const uint4* q = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.x) + (int64_t)b * p.sB +
                                                  (int64_t)t * p.sT + col);
#pragma unroll
  for (int j = 0; j < RawBlock<DT>::NV; ++j) r.u[j] = __ldg(q + j);
}

template <int DT, int A>
__device__ __forceinline__ void unpack_raw(float v[16], const RawBlock<DT>& r) {
#pragma unroll
  for (int j = 0; j < RawBlock<DT>::NV; ++j) {
    const uint32_t w[4] = {r.u[j].x, r.u[j].y, r.u[j].z, r.u[j].w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if constexpr (DT == FP4_DT_F32) {
        v[4 * j + k] = rnd<A>(__uint_as_float(w[k]));
      } else if constexpr (DT == FP4_DT_BF16) {
        v[8 * j + 2 * k] = rnd<A>(__uint_as_float(w[k] << 16));
        v[8 * j + 2 * k + 1] = rnd<A>(__uint_as_float(w[k] & 0xFFFF0000u));
      } else {
        const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
        v[8 * j + 2 * k] = rnd<A>(f2.x);
        v[8 * j + 2 * k + 1] = rnd<A>(f2.y);
      }
    }
  }
}

// Persistent row quantizer for aligned rows of whole 16-element blocks
// (n % 16 == 0, every block 16-byte aligned) with at most 2 blocks per
// thread: each CTA walks row groups with a grid stride and loads the next
// group's raw vectors before it quantizes the current one, so a thread keeps
// one row's bytes in flight while it computes.  Same arithmetic as
// quant_rows_kernel (quant_block).
// x - (code * s) * g for the 16 values of a block quantized to (w, s) under g:
// the residual dual_nvfp4 quantizes second (fp4_quant_utils.py:313-315).
template <int A>
__device__ __forceinline__ void block_residual(float v[16], const uint32_t w[2], float s, float g) {
#pragma unroll
  for (int j = 0; j < 16; ++j)
    v[j] = __fsub_rn(v[j], mul<A>(mul<A>(e2m1_value((w[j >> 3] >> (4 * (j & 7))) & 15u), s), g));
}

// DUAL (row mode only): after the first slice, the same row-mode quantizer
// runs on the fp32 residual x - dequant(first slice), held in registers as
// the raw block and the first slice's codes, into codes_lo / scales_lo / g_row_lo.
template <int DT, int A, int ODT, int TPR, bool OUT, bool DUAL = false>
__global__ void __launch_bounds__(kVecThreads, 3) quant_rows_vec_kernel(QuantArgs p) {
  constexpr int ROWS = kVecThreads / TPR;
  constexpr int WPR = TPR / 32;
  __shared__ float red[2][kVecThreads / 32];
  __shared__ float red2[2][kVecThreads / 32];
  __shared__ float rcp_tab[128];
  if (threadIdx.x < 128) rcp_tab[threadIdx.x] = recip<A>(e4m3_to_f32((uint8_t)threadIdx.x));
  __syncthreads();
  const int rloc = threadIdx.x / TPR;
  const int lane = threadIdx.x % TPR;
  const int64_t nrows = (int64_t)p.B * p.T_pad;
  const int nblk = p.H * p.D / 16;
  const int nmine = lane < nblk ? (nblk - lane + TPR - 1) / TPR : 0;  // 0, 1 or 2
  const int64_t step = (int64_t)gridDim.x * ROWS;
  // a thread's blocks sit at the same columns of every row
  const int64_t col0 = block_col_offset(p, lane), col1 = block_col_offset(p, lane + TPR);
  const uint32_t tpad = (uint32_t)p.T_pad;
  auto row_bt = [&](int64_t orow, int& b, int& t) {
    if (p.B == 1) {
      b = 0;
      t = (int)orow;
    } else {
      b = (int)((uint32_t)orow / tpad);
      t = (int)((uint32_t)orow - (uint32_t)b * tpad);
    }
  };
  // tensor mode: the one global scale and its reciprocal, read and computed once
  const float g_tensor = p.gmode == 3 ? p.g_in[0] : 1.0f;
  const float rg_tensor = p.gmode == 3 ? recip<A>(g_tensor) : 1.0f;
  RawBlock<DT> cur[2], nxt[2];
  uint32_t whi[2][2] = {{0u, 0u}, {0u, 0u}};  // DUAL: first-slice codes and scales of this thread's blocks
  float shi[2] = {0.0f, 0.0f};
  int64_t base = (int64_t)blockIdx.x * ROWS;
  {
    const int64_t orow = base + rloc;
    int b, t;
    row_bt(orow, b, t);
    if (orow < nrows && t < p.T) {
#pragma unroll
      for (int i = 0; i < 2; ++i)
        if (i < nmine) load_raw<DT>(cur[i], p, b, t, i ? col1 : col0);
    }
  }
  for (int it = 0; base < nrows; base += step, ++it) {
    const int64_t orow = base + rloc;
    const bool live = orow < nrows;
    int b = 0, t = 0;
    if (live) row_bt(orow, b, t);
    const bool pad_row = !live || t >= p.T;
    {  // the next row group's bytes go in flight now
      const int64_t nrow = orow + step;
      int nb, nt;
      row_bt(nrow, nb, nt);
      if (nrow < nrows && nt < p.T) {
#pragma unroll
        for (int i = 0; i < 2; ++i)
          if (i < nmine) load_raw<DT>(nxt[i], p, nb, nt, i ? col1 : col0);
      }
    }
    float g = 1.0f;
    if (p.gmode == 1) {
      float m = 0.0f;
      if (!pad_row) {
#pragma unroll
        for (int i = 0; i < 2; ++i)
          if (i < nmine) {
            float v[16];
            unpack_raw<DT, A>(v, cur[i]);
            m = nanmax(m, block_absmax(v));
          }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = nanmax(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (WPR > 1) {
        if ((threadIdx.x & 31) == 0) red[it & 1][threadIdx.x / 32] = m;
        __syncthreads();
        m = red[it & 1][rloc * WPR];
#pragma unroll
        for (int w = 1; w < WPR; ++w) m = nanmax(m, red[it & 1][rloc * WPR + w]);
      }
      g = m;  // rowmax, no division by global_sf_max (fp4_quant_utils.py:134,139)
      if (p.g_row && lane == 0 && live) p.g_row[orow] = pad_row ? 0.0f : g;
    } else if (p.gmode == 3) {
      g = g_tensor;
    }
    if (live) {
      if (pad_row) {
        for (int kb = lane; kb < nblk; kb += TPR) {
          if (p.codes) *reinterpret_cast<uint2*>(p.codes + orow * p.codes_ld + (int64_t)kb * 8) = make_uint2(0u, 0u);
          if (p.scales)
            p.scales[p.scale_layout ? sf_tcgen05_offset(orow, kb, p.scales_ld) : orow * p.scales_ld + kb] = 0;
        }
      } else {
        const float rg = p.gmode == 0 ? 1.0f : p.gmode == 3 ? rg_tensor : recip<A>(g);
#pragma unroll
        for (int i = 0; i < 2; ++i)
          if (i < nmine) {
            float v[16];
            unpack_raw<DT, A>(v, cur[i]);
            if constexpr (DUAL) quant_block<A, ODT, false, OUT>(v, p, orow, lane + i * TPR, g, rg, rcp_tab, whi[i], &shi[i]);
            else quant_block<A, ODT, false, OUT>(v, p, orow, lane + i * TPR, g, rg, rcp_tab);
          }
      }
    }
    if constexpr (DUAL) {
      float m = 0.0f;
      if (!pad_row) {
#pragma unroll
        for (int i = 0; i < 2; ++i)
          if (i < nmine) {
            float v[16];
            unpack_raw<DT, A>(v, cur[i]);
            block_residual<A>(v, whi[i], shi[i], g);
            m = nanmax(m, block_absmax(v));
          }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = nanmax(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (WPR > 1) {
        if ((threadIdx.x & 31) == 0) red2[it & 1][threadIdx.x / 32] = m;
        __syncthreads();
        m = red2[it & 1][rloc * WPR];
#pragma unroll
        for (int w = 1; w < WPR; ++w) m = nanmax(m, red2[it & 1][rloc * WPR + w]);
      }
      const float g2 = m;
      if (p.g_row_lo && lane == 0 && live) p.g_row_lo[orow] = pad_row ? 0.0f : g2;
      if (live) {
        QuantArgs pl = p;
        pl.codes = p.codes_lo;
        pl.scales = p.scales_lo;
        if (pad_row) {
          for (int kb = lane; kb < nblk; kb += TPR) {
            *reinterpret_cast<uint2*>(pl.codes + orow * pl.codes_ld + (int64_t)kb * 8) = make_uint2(0u, 0u);
            pl.scales[pl.scale_layout ? sf_tcgen05_offset(orow, kb, pl.scales_ld) : orow * pl.scales_ld + kb] = 0;
          }
        } else {
          const float rg2 = recip<A>(g2);
#pragma unroll
          for (int i = 0; i < 2; ++i)
            if (i < nmine) {
              float v[16];
              unpack_raw<DT, A>(v, cur[i]);
              block_residual<A>(v, whi[i], shi[i], g);
              quant_block<A, ODT, false, false>(v, pl, orow, lane + i * TPR, g2, rg2, rcp_tab);
            }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) cur[i] = nxt[i];
  }
}

// Dual-slice row mode (fp32 arithmetic) on the persistent row kernel; -1 when
// the layout is not one it takes (unaligned rows, more than 512 blocks a row).
template <int DT>
static int launch_rows_dual(const QuantArgs& p, cudaStream_t st) {
  constexpr int A = FP4_ARITH_F32;
  const int64_t n = (int64_t)p.H * p.D;
  const int64_t nblk = (n + 15) / 16;
  const int64_t nrows = (int64_t)p.B * p.T_pad;
  if (!(p.vec && n % 16 == 0 && nblk <= 256 * 2 && (p.H == 1 || p.D % 16 == 0))) return -1;
  const int tpr = nblk <= 64 ? 32 : nblk <= 128 ? 64 : nblk <= 256 ? 128 : 256;
  const int64_t groups = (nrows + (kVecThreads / tpr) - 1) / (kVecThreads / tpr);
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(groups, 148 * 3));
  switch (tpr) {
    case 32: quant_rows_vec_kernel<DT, A, A, 32, false, true><<<grid, kVecThreads, 0, st>>>(p); break;
    case 64: quant_rows_vec_kernel<DT, A, A, 64, false, true><<<grid, kVecThreads, 0, st>>>(p); break;
    case 128: quant_rows_vec_kernel<DT, A, A, 128, false, true><<<grid, kVecThreads, 0, st>>>(p); break;
    default: quant_rows_vec_kernel<DT, A, A, 256, false, true><<<grid, kVecThreads, 0, st>>>(p); break;
  }
  return check_launch("quant_rows_vec_kernel(dual)");
}

template <int DT, int A, int ODT, bool COLG, bool OUT>
static int launch_rows(const QuantArgs& p, cudaStream_t st) {
  const int64_t n = (int64_t)p.H * p.D;
  const int64_t nblk = (n + 15) / 16;
  const int64_t nrows = (int64_t)p.B * p.T_pad;
  if constexpr (!COLG) {
    if (p.vec && n % 16 == 0 && nblk <= 256 * 2 && (p.H == 1 || p.D % 16 == 0)) {
      // persistent: a few CTAs per SM, each walking row groups
      int tpr = nblk <= 64 ? 32 : nblk <= 128 ? 64 : nblk <= 256 ? 128 : 256;
      const int64_t groups = (nrows + (kVecThreads / tpr) - 1) / (kVecThreads / tpr);
      const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(groups, 148 * 3));
      switch (tpr) {
        case 32: quant_rows_vec_kernel<DT, A, ODT, 32, OUT><<<grid, kVecThreads, 0, st>>>(p); break;
        case 64: quant_rows_vec_kernel<DT, A, ODT, 64, OUT><<<grid, kVecThreads, 0, st>>>(p); break;
        case 128: quant_rows_vec_kernel<DT, A, ODT, 128, OUT><<<grid, kVecThreads, 0, st>>>(p); break;
        default: quant_rows_vec_kernel<DT, A, ODT, 256, OUT><<<grid, kVecThreads, 0, st>>>(p); break;
      }
      return check_launch("quant_rows_vec_kernel");
    }
  }
  // threads per row: enough that each thread owns at most MAXB blocks when possible
  if (nblk <= 32 * MAXB) {
    quant_rows_kernel<DT, A, ODT, 32, COLG, OUT><<<(unsigned)((nrows + 3) / 4), kThreads, 0, st>>>(p);
  } else if (nblk <= 64 * MAXB) {
    quant_rows_kernel<DT, A, ODT, 64, COLG, OUT><<<(unsigned)((nrows + 1) / 2), kThreads, 0, st>>>(p);
  } else {
    quant_rows_kernel<DT, A, ODT, 128, COLG, OUT><<<(unsigned)nrows, kThreads, 0, st>>>(p);
  }
  return check_launch("quant_rows_kernel");
}

template <int DT, int A>
static int launch_prepass(const QuantArgs& p, float* g, float gsf_max, cudaStream_t st) {
  const int64_t n = (int64_t)p.H * p.D;
  const int64_t npad = (n + 15) / 16 * 16;
  const int per_col = p.gmode == 2;
  const int64_t count = per_col ? npad : 1;
  if (cudaMemsetAsync(g, 0, count * sizeof(float), st) != cudaSuccess) return set_error(FP4ATTN_ERR_CUDA, "memset g");
  const int64_t nrows = (int64_t)p.B * p.T;
  // A contiguous tensor in tensor mode is one flat run of elements.
  const bool flat = !per_col && p.vec && (p.H == 1 || p.sH == p.D) && p.sT == n && (p.B == 1 || p.sB == (int64_t)p.T * n);
  if (flat) {
    const int64_t nelem = nrows * n;
    const int64_t chunks = nelem / (16 / (int64_t)sizeof(typename In<DT>::T));
    // about eight chunks per thread: one batch of loads each
    const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>(148 * 8, (chunks + 2047) / 2048));
    absmax_flat_kernel<DT, A><<<blocks, 256, 0, st>>>(p.x, nelem, reinterpret_cast<unsigned int*>(g));
    if (int e = check_launch("absmax_flat_kernel")) return e;
    finalize_g_kernel<A><<<1, 32, 0, st>>>(g, count, gsf_max);
    return check_launch("finalize_g_kernel");
  }
  const unsigned gx = (unsigned)((n + 8 * 256 - 1) / (8 * 256));
  // Enough row slices to fill the GPU several times over.
  unsigned gy = (unsigned)std::max<int64_t>(1, std::min<int64_t>(nrows, (148 * 16 + gx - 1) / gx));
  absmax_kernel<DT, A><<<dim3(gx, gy), 256, 0, st>>>(p, reinterpret_cast<unsigned int*>(g), per_col);
  if (int e = check_launch("absmax_kernel")) return e;
  finalize_g_kernel<A><<<(unsigned)((count + 255) / 256), 256, 0, st>>>(g, count, gsf_max);
  return check_launch("finalize_g_kernel");
}

template <int DT, int A, int ODT>
static int run_quant(QuantArgs p, float* g, float gsf_max, bool g_ready, cudaStream_t st) {
  if (p.gmode == 2 || p.gmode == 3) {
    if (!g_ready)
      if (int e = launch_prepass<DT, A>(p, g, gsf_max, st)) return e;
    p.g_in = g;
  } else if (p.gmode == 1) {
    p.g_row = g;
  }
  const bool colg = p.gmode == 2, out = p.out != nullptr;
  if (colg) return out ? launch_rows<DT, A, ODT, true, true>(p, st) : launch_rows<DT, A, ODT, true, false>(p, st);
  return out ? launch_rows<DT, A, ODT, false, true>(p, st) : launch_rows<DT, A, ODT, false, false>(p, st);
}

// what: 0 = full quantize (reduction + rows), 1 = rows with g ready, 2 = reduction only.
template <int DT, int A>
static int dispatch_odt(const QuantArgs& p, int out_dtype, float* g, float gsf_max, int what, cudaStream_t st) {
  if (what == 2) return launch_prepass<DT, A>(p, g, gsf_max, st);
  const bool ready = what == 1;
  if (p.out && out_dtype != A) return set_error(FP4ATTN_ERR_UNSUPPORTED, "out_dtype must equal the dequant dtype");
  return run_quant<DT, A, A>(p, g, gsf_max, ready, st);
}

template <int DT>
static int dispatch_arith(const QuantArgs& p, int arith, int out_dtype, float* g, float gsf_max, int what,
                          cudaStream_t st) {
  switch (arith) {
    case FP4_ARITH_F32: return dispatch_odt<DT, FP4_ARITH_F32>(p, out_dtype, g, gsf_max, what, st);
    case FP4_ARITH_BF16: return dispatch_odt<DT, FP4_ARITH_BF16>(p, out_dtype, g, gsf_max, what, st);
    case FP4_ARITH_F16: return dispatch_odt<DT, FP4_ARITH_F16>(p, out_dtype, g, gsf_max, what, st);
  }
  return set_error(FP4ATTN_ERR_ARG, "bad arith");
}

// Single-pass per-tensor quantize (quant_fused.cu); -1 when not applicable.
int quant_tensor_fused(const void* x, int in_dtype, int64_t nelem, uint8_t* codes, uint8_t* scales, float* g,
                       float gsf_max, cudaStream_t st);
unsigned int quant_status(bool reset);

// One instantiation set per input dtype (quant_f32.cu, quant_bf16.cu, quant_f16.cu).
int quant_dispatch_f32(const QuantArgs& p, int arith, int out_dtype, float* g, float gsf_max, int what, cudaStream_t st);
int quant_dispatch_bf16(const QuantArgs& p, int arith, int out_dtype, float* g, float gsf_max, int what, cudaStream_t st);
int quant_dispatch_f16(const QuantArgs& p, int arith, int out_dtype, float* g, float gsf_max, int what, cudaStream_t st);
// dual-slice row mode (launch_rows_dual); -1 when the layout is not supported
int quant_dual_f32(const QuantArgs& p, cudaStream_t st);
int quant_dual_bf16(const QuantArgs& p, cudaStream_t st);
int quant_dual_f16(const QuantArgs& p, cudaStream_t st);

}  // namespace fp4
