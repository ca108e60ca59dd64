// quant.cu -- C ABI entry points of the NVFP4 quantizer (fp4q_quantize,
// fp4q_global_scale).  The kernels live in quant_impl.cuh.
#include <stdint.h>

#include "quant_impl.cuh"

using namespace fp4;

static int quantize_entry(const void* x, int in_dtype, int B, int T, int H, int D, int64_t sB, int64_t sT,
                          int64_t sH, int T_pad, int gmode, int arith, float global_sf_max, uint8_t* codes,
                          int64_t codes_ld, uint8_t* scales, int scale_layout, int64_t scales_ld, float* g, void* out,
                          int out_dtype, int64_t out_ld, void* stream, int what) {
  clear_error();
  if (!x) return set_error(FP4ATTN_ERR_ARG, "x is null");
  if (B <= 0 || T < 0 || H <= 0 || D <= 0 || T_pad < T) return set_error(FP4ATTN_ERR_ARG, "bad shape");
  // rows and columns are indexed in 32 bits inside the kernels
  if ((int64_t)H * D > INT32_MAX || (int64_t)B * T_pad > INT32_MAX)
    return set_error(FP4ATTN_ERR_ARG, "rows (B*T_pad) and columns (H*D) must each be below 2^31");
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
  // Per-tensor mode on a contiguous tensor that fits on chip: one pass over HBM.
  if (what == 0 && gmode == 3 && arith == FP4_ARITH_F32 && !out && codes && scales && scale_layout == 0 &&
      p.vec && T_pad == T) {
    const int64_t n = (int64_t)H * D;
    const bool flat = (H == 1 || sH == D) && sT == n && (B == 1 || sB == (int64_t)T * n);
    if (flat && n % 16 == 0 && codes_ld == n / 2 && scales_ld == n / 16) {
      const int r = quant_tensor_fused(x, in_dtype, (int64_t)B * T * n, codes, scales, g, global_sf_max, st);
      if (r >= 0) return r;
    }
  }
  switch (in_dtype) {
    case FP4_DT_F32: return quant_dispatch_f32(p, arith, out_dtype, g, global_sf_max, what, st);
    case FP4_DT_BF16: return quant_dispatch_bf16(p, arith, out_dtype, g, global_sf_max, what, st);
    case FP4_DT_F16: return quant_dispatch_f16(p, arith, out_dtype, g, global_sf_max, what, st);
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

extern "C" int fp4q_quantize_dual(const void* x, int in_dtype, int B, int T, int H, int D, int64_t sB, int64_t sT,
                                  int64_t sH, int T_pad, uint8_t* codes, int64_t codes_ld, uint8_t* scales,
                                  int scale_layout, int64_t scales_ld, float* g, uint8_t* codes_lo, uint8_t* scales_lo,
                                  float* g_lo, void* stream) {
  clear_error();
  if (!x || !codes || !scales || !g || !codes_lo || !scales_lo || !g_lo) return set_error(FP4ATTN_ERR_ARG, "null pointer");
  if (B <= 0 || T < 0 || H <= 0 || D <= 0 || T_pad < T) return set_error(FP4ATTN_ERR_ARG, "bad shape");
  if ((int64_t)H * D > INT32_MAX || (int64_t)B * T_pad > INT32_MAX)
    return set_error(FP4ATTN_ERR_ARG, "rows (B*T_pad) and columns (H*D) must each be below 2^31");
  if (H > 1 && D % 16 != 0) return set_error(FP4ATTN_ERR_ARG, "D must be a multiple of 16 when H > 1");
  if (scale_layout == 1 && T_pad % 128 != 0 && B > 1)
    return set_error(FP4ATTN_ERR_ARG, "tcgen05 scale layout needs T_pad % 128 == 0");
  if (codes_ld % 8 != 0) return set_error(FP4ATTN_ERR_ARG, "codes_ld must be a multiple of 8");
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
  p.gmode = 1;
  p.g_row = g;
  p.codes = codes;
  p.codes_ld = codes_ld;
  p.scales = scales;
  p.scale_layout = scale_layout;
  p.scales_ld = scales_ld;
  p.codes_lo = codes_lo;
  p.scales_lo = scales_lo;
  p.g_row_lo = g_lo;
  const bool aligned = ((uintptr_t)x % 16 == 0) && ((sB * esz) % 16 == 0 || B == 1) && ((sT * esz) % 16 == 0 || T == 1) &&
                       ((sH * esz) % 16 == 0 || H == 1) && ((D * esz) % 16 == 0 || H == 1);
  p.vec = aligned ? 1 : 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int r = -1;
  switch (in_dtype) {
    case FP4_DT_F32: r = quant_dual_f32(p, st); break;
    case FP4_DT_BF16: r = quant_dual_bf16(p, st); break;
    case FP4_DT_F16: r = quant_dual_f16(p, st); break;
    default: return set_error(FP4ATTN_ERR_ARG, "bad in_dtype");
  }
  if (r < 0)
    return set_error(FP4ATTN_ERR_UNSUPPORTED,
                     "dual quantize needs 16-byte aligned rows of whole 16-blocks, at most 8192 columns");
  return r;
}
