// quant.cu -- NVFP4 quantize / fused quantize-dequantize kernels (sm_100a).
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
#include <stdio.h>

#include <algorithm>

#include "common.cuh"
#include "status.h"

namespace fp4 {

constexpr int kThreads = 128;
constexpr int MAXB = 4;

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
};

template <int DT, int A>
__device__ __forceinline__ void load_block(float v[16], const QuantArgs& p, int b, int t, int kb) {
  using T = typename In<DT>::T;
  const int64_t n = (int64_t)p.H * p.D;
  const int64_t c0 = (int64_t)kb * 16;
  const T* base = reinterpret_cast<const T*>(p.x) + (int64_t)b * p.sB + (int64_t)t * p.sT;
  if (p.vec && c0 + 16 <= n) {
    const int h = (int)(c0 / p.D);
    const int d = (int)(c0 - (int64_t)h * p.D);
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
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[8 * j + k] = rnd<A>(In<DT>::f(e[k]));
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

// Quantize one block (values already in the dequant dtype, before the global
// scale) and write codes / scale byte / dequantized values.
template <int A, int ODT>
__device__ __forceinline__ void quant_block(float v[16], const QuantArgs& p, int64_t orow, int kb, float g, float rg,
                                           const float* gcol) {
  const int64_t n = (int64_t)p.H * p.D;
  const float r6 = recip<A>(6.0f);
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (p.gmode == 2) {
      v[j] = mul<A>(v[j], recip<A>(gcol[kb * 16 + j]));
    } else if (p.gmode != 0) {
      v[j] = mul<A>(v[j], rg);
    }
    amax = nanmax(amax, fabsf(v[j]));
  }
  const uint8_t sb = e4m3_torch(mul<A>(amax, r6));
  const float s = e4m3_to_f32(sb);
  const float rs = recip<A>(s);
  const bool nan_block = (sb & 0x7F) == 0x7F;
  uint32_t w[2] = {0u, 0u};
  float q[16];
#pragma unroll
  for (int j = 0; j < 16; j += 2) {
    // + 0.0f turns -0.0 into +0.0: torch.sign(-0.0) is 0 (fp4_quant_utils.py:49,62).
    const float a = mul<A>(v[j], rs) + 0.0f;
    const float c = mul<A>(v[j + 1], rs) + 0.0f;
    uint32_t byte = nan_block ? 0u : e2m1x2(a, c);
    w[j >> 3] |= byte << (4 * (j & 7));
    q[j] = e2m1_value(byte & 15u);
    q[j + 1] = e2m1_value(byte >> 4);
  }
  if (p.codes) {
    *reinterpret_cast<uint2*>(p.codes + orow * p.codes_ld + (int64_t)kb * 8) = make_uint2(w[0], w[1]);
  }
  if (p.scales) {
    const int64_t off = p.scale_layout ? sf_tcgen05_offset(orow, kb, p.scales_ld) : orow * p.scales_ld + kb;
    p.scales[off] = sb;
  }
  if (p.out) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int64_t c = (int64_t)kb * 16 + j;
      if (c < n) {
        float o = mul<A>(q[j], s);
        if (p.gmode == 2) o = mul<A>(o, gcol[c]);
        else if (p.gmode != 0) o = mul<A>(o, g);
        store_out<ODT>(p.out, orow * p.out_ld + c, o);
      }
    }
  }
}

template <int DT, int A, int ODT, int TPR>
__global__ void __launch_bounds__(kThreads) quant_rows_kernel(QuantArgs p) {
  constexpr int ROWS = kThreads / TPR;
  constexpr int WPR = TPR / 32;  // warps per row
  __shared__ float red[kThreads / 32];
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

  float cache[MAXB][16];
  float g = 0.0f;
  if (p.gmode == 1) {
    float m = 0.0f;
    if (!pad_row) {
      int i = 0;
      for (int kb = lane; kb < nblk; kb += TPR, ++i) {
        float v[16];
        load_block<DT, A>(v, p, b, t, kb);
#pragma unroll
        for (int j = 0; j < 16; ++j) m = nanmax(m, fabsf(v[j]));
        if (i < MAXB) {
#pragma unroll
          for (int j = 0; j < 16; ++j) cache[i][j] = v[j];
        }
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
  const float rg = recip<A>(g);
  int i = 0;
  for (int kb = lane; kb < nblk; kb += TPR, ++i) {
    float v[16];
    if (p.gmode == 1 && i < MAXB) {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = cache[i][j];
    } else {
      load_block<DT, A>(v, p, b, t, kb);
    }
    quant_block<A, ODT>(v, p, orow, kb, g, rg, p.g_in);
  }
}

// Column / tensor maxima of |x| (in the dequant dtype) into bits[].
template <int DT, int A>
__global__ void __launch_bounds__(256) absmax_kernel(QuantArgs p, unsigned int* bits, int per_column) {
  const int64_t n = (int64_t)p.H * p.D;
  const int64_t nrows = (int64_t)p.B * p.T;
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t rows_per = (nrows + gridDim.y - 1) / gridDim.y;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per;
  const int64_t r1 = r0 + rows_per < nrows ? r0 + rows_per : nrows;
  float m = 0.0f;
  if (c < n) {
    using T = typename In<DT>::T;
    const int h = (int)(c / p.D);
    const int d = (int)(c - (int64_t)h * p.D);
    for (int64_t r = r0; r < r1; ++r) {
      const int b = (int)(r / p.T);
      const int t = (int)(r - (int64_t)b * p.T);
      const T* q = reinterpret_cast<const T*>(p.x) + (int64_t)b * p.sB + (int64_t)t * p.sT + (int64_t)h * p.sH + d;
      m = nanmax(m, fabsf(rnd<A>(In<DT>::f(*q))));
    }
  }
  if (per_column) {
    if (c < n && r1 > r0) atomicMax(bits + c, __float_as_uint(m));
    return;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = nanmax(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(bits, __float_as_uint(m));
}

// g = max * recip(global_sf_max) in the dequant dtype (fp4_quant_utils.py:139).
template <int A>
__global__ void finalize_g_kernel(float* g, int64_t count, float gsf_max) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) g[i] = mul<A>(g[i], recip<A>(rnd<A>(gsf_max)));
}

template <int DT, int A, int ODT>
static int launch_rows(const QuantArgs& p, cudaStream_t st) {
  const int64_t n = (int64_t)p.H * p.D;
  const int64_t nblk = (n + 15) / 16;
  const int64_t nrows = (int64_t)p.B * p.T_pad;
  if (nblk <= 32) {
    quant_rows_kernel<DT, A, ODT, 32><<<(unsigned)((nrows + 3) / 4), kThreads, 0, st>>>(p);
  } else if (nblk <= 64) {
    quant_rows_kernel<DT, A, ODT, 64><<<(unsigned)((nrows + 1) / 2), kThreads, 0, st>>>(p);
  } else {
    quant_rows_kernel<DT, A, ODT, 128><<<(unsigned)nrows, kThreads, 0, st>>>(p);
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
  const unsigned gx = (unsigned)((n + 255) / 256);
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
  return launch_rows<DT, A, ODT>(p, st);
}

// what: 0 = full quantize (reduction + rows), 1 = rows with g ready, 2 = reduction only.
template <int DT, int A>
static int dispatch_odt(const QuantArgs& p, int out_dtype, float* g, float gsf_max, int what, cudaStream_t st) {
  if (what == 2) return launch_prepass<DT, A>(p, g, gsf_max, st);
  const bool ready = what == 1;
  switch (out_dtype) {
    case FP4_DT_F32: return run_quant<DT, A, FP4_DT_F32>(p, g, gsf_max, ready, st);
    case FP4_DT_BF16: return run_quant<DT, A, FP4_DT_BF16>(p, g, gsf_max, ready, st);
    case FP4_DT_F16: return run_quant<DT, A, FP4_DT_F16>(p, g, gsf_max, ready, st);
  }
  return set_error(FP4ATTN_ERR_ARG, "bad out_dtype");
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

}  // namespace fp4

using namespace fp4;

static int quantize_entry(const void* x, int in_dtype, int B, int T, int H, int D, int64_t sB, int64_t sT,
                          int64_t sH, int T_pad, int gmode, int arith, float global_sf_max, uint8_t* codes,
                          int64_t codes_ld, uint8_t* scales, int scale_layout, int64_t scales_ld, float* g, void* out,
                          int out_dtype, int64_t out_ld, void* stream, int what) {
  clear_error();
  if (!x) return set_error(FP4ATTN_ERR_ARG, "x is null");
  if (B <= 0 || T < 0 || H <= 0 || D <= 0 || T_pad < T) return set_error(FP4ATTN_ERR_ARG, "bad shape");
  if (H > 1 && D % 16 != 0) return set_error(FP4ATTN_ERR_ARG, "D must be a multiple of 16 when H > 1");
  if (gmode < 0 || gmode > 3) return set_error(FP4ATTN_ERR_ARG, "bad gmode");
  if (gmode != 0 && !g) return set_error(FP4ATTN_ERR_ARG, "g buffer required for a global-scale mode");
  if (what == 2 && gmode != 2 && gmode != 3) return set_error(FP4ATTN_ERR_ARG, "global-scale pass needs gmode 2 or 3");
  if (gmode == 2 && H != 1) return set_error(FP4ATTN_ERR_ARG, "column mode needs a 2-D input (H == 1)");
  if (scale_layout == 1 && T_pad % 128 != 0 && B > 1)
    return set_error(FP4ATTN_ERR_ARG, "tcgen05 scale layout needs T_pad % 128 == 0");
  if (codes && (codes_ld % 8 != 0)) return set_error(FP4ATTN_ERR_ARG, "codes_ld must be a multiple of 8");
  if (T == 0) return FP4ATTN_OK;
  const int64_t esz = in_dtype == FP4_DT_F32 ? 4 : 2;
  QuantArgs p{};
  p.x = x;
  p.sB = sB;
  p.sT = sT;
  p.sH = sH;
  p.B = B;
  p.T = T;
  p.H = H;
  p.D = D;
  p.T_pad = T_pad;
  p.gmode = gmode;
  p.codes = codes;
  p.codes_ld = codes_ld;
  p.scales = scales;
  p.scale_layout = scale_layout;
  p.scales_ld = scales_ld;
  p.out = out;
  p.out_ld = out_ld;
  // Vector loads need every 16-element block start 16-byte aligned.
  const bool aligned = ((uintptr_t)x % 16 == 0) && ((sB * esz) % 16 == 0 || B == 1) && ((sT * esz) % 16 == 0 || T == 1) &&
                       ((sH * esz) % 16 == 0 || H == 1) && ((D * esz) % 16 == 0 || H == 1);
  p.vec = aligned ? 1 : 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (in_dtype) {
    case FP4_DT_F32: return dispatch_arith<FP4_DT_F32>(p, arith, out_dtype, g, global_sf_max, what, st);
    case FP4_DT_BF16: return dispatch_arith<FP4_DT_BF16>(p, arith, out_dtype, g, global_sf_max, what, st);
    case FP4_DT_F16: return dispatch_arith<FP4_DT_F16>(p, arith, out_dtype, g, global_sf_max, what, st);
  }
  return set_error(FP4ATTN_ERR_ARG, "bad in_dtype");
}

extern "C" int fp4q_quantize(const void* x, int in_dtype, int B, int T, int H, int D, int64_t sB, int64_t sT,
                             int64_t sH, int T_pad, int gmode, int arith, float global_sf_max, uint8_t* codes,
                             int64_t codes_ld, uint8_t* scales, int scale_layout, int64_t scales_ld, float* g,
                             void* out, int out_dtype, int64_t out_ld, void* stream) {
  const int ready = (gmode & 0x10) ? 1 : 0;
  return quantize_entry(x, in_dtype, B, T, H, D, sB, sT, sH, T_pad, gmode & 0xF, arith, global_sf_max, codes,
                        codes_ld, scales, scale_layout, scales_ld, g, out, out_dtype, out_ld, stream, ready);
}

extern "C" int fp4q_global_scale(const void* x, int in_dtype, int B, int T, int H, int D, int64_t sB, int64_t sT,
                                 int64_t sH, int gmode, int arith, float global_sf_max, float* g, void* stream) {
  return quantize_entry(x, in_dtype, B, T, H, D, sB, sT, sH, T, gmode, arith, global_sf_max, nullptr, 0, nullptr, 0,
                        0, g, nullptr, 0, 0, stream, 2);
}
