// attn_decode.cu -- FP4 attention for one new query token per sequence over an
// NVFP4 KV cache (decode).
//
// The reference's patched attention (llama_patch.py:167-215) quantizes each
// call's new Q/K/V, appends the dequantized K/V to the HF cache and runs the
// eager attention with P fake-quant (llama_patch.py:57-105) over every cached
// key.  Here the cache holds the packed NVFP4 data of those same values:
//   K: codes [B][Hkv][Tmax][D/2], E4M3 scales per 16 dims [B][Hkv][Tmax][D/16],
//      per-token global scale g_k [B][Tmax] (row mode on the [B*q, Hkv*D] view);
//   V: codes [B][Hkv][Tmax][D/2], one E4M3 scale byte per element
//      [B][Hkv][Tmax][D] (V's blocks of 16 run along the tokens of the call that
//      appended them, so a token's scale is per channel), per-token g_v [B][Tmax].
// The query is passed already fake-quantized (Q-hat, fp32 [B][Hq][D]).
//
// Three kernels, all HBM-bound: scores S = Q-hat K-hat^T * scaling per split of
// keys (with the split's row maxima); then the exact row max, e =
// exp2((S - m) log2 e), the NVFP4 fake-quant of e per 16 keys (as the prefill
// kernel does) and O-partial = P-hat V-hat on CUDA cores; then the combine
// O = sum O-partial / sum l.
#include <stdint.h>

#include "common.cuh"
#include "fp4attn.h"
#include "status.h"

namespace fp4 {
namespace {

constexpr int DK_KEYS = 256;     // keys per split (one per thread in the score kernel)
constexpr int DK_MAXG = 16;      // query heads per KV head
constexpr int DK_D = 128;        // head dim

struct DecodeArgs {
  const float* qhat;  // [B][Hq][D]
  const uint8_t* k_codes;
  const uint8_t* k_scales;
  const float* k_g;
  const uint8_t* v_codes;
  const uint8_t* v_scales;
  const float* v_g;
  int B, Hq, Hkv, len, Tmax, nsplit;
  float scaling;
  float* S;      // [B][Hq][nsplit*DK_KEYS]
  float* pmax;   // [B][Hq][nsplit]
  float* opart;  // [B][Hq][nsplit][D]
  float* lpart;  // [B][Hq][nsplit]
  float* out;    // [B][Hq][D]
};

__global__ void __launch_bounds__(DK_KEYS) decode_scores_kernel(DecodeArgs p) {
  const int split = blockIdx.x, bk = blockIdx.y;
  const int b = bk / p.Hkv, hk = bk % p.Hkv;
  const int G = p.Hq / p.Hkv;
  __shared__ float q_s[DK_MAXG][DK_D];
  __shared__ float red[DK_KEYS / 32][DK_MAXG];
  for (int i = threadIdx.x; i < G * DK_D; i += DK_KEYS)
    q_s[i / DK_D][i % DK_D] = p.qhat[((int64_t)b * p.Hq + hk * G + i / DK_D) * DK_D + i % DK_D];
  __syncthreads();
  const int k = split * DK_KEYS + threadIdx.x;
  float acc[DK_MAXG];
#pragma unroll
  for (int g = 0; g < DK_MAXG; ++g) acc[g] = 0.0f;
  const bool live = k < p.len;
  if (live) {
    const int64_t row = ((int64_t)b * p.Hkv + hk) * p.Tmax + k;
    const uint4* c4 = reinterpret_cast<const uint4*>(p.k_codes + row * (DK_D / 2));
    const uint2 sc = *reinterpret_cast<const uint2*>(p.k_scales + row * (DK_D / 16));
    const uint8_t* sb = reinterpret_cast<const uint8_t*>(&sc);
#pragma unroll
    for (int w = 0; w < 4; ++w) {  // 32 dims per 16-byte word
      const uint4 u = c4[w];
      const uint32_t words[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const int d = w * 32 + j * 8 + n;
          const float kv = __fmul_rn(e2m1_value((words[j] >> (4 * n)) & 15u), e4m3_to_f32(sb[d / 16]));
#pragma unroll
          for (int g = 0; g < DK_MAXG; ++g)
            if (g < G) acc[g] = __fmaf_rn(q_s[g][d], kv, acc[g]);
        }
      }
    }
    const float gk = p.k_g[(int64_t)b * p.Tmax + k];
#pragma unroll
    for (int g = 0; g < DK_MAXG; ++g) acc[g] = __fmul_rn(__fmul_rn(acc[g], gk), p.scaling);
  }
  const int ks = p.nsplit * DK_KEYS;
#pragma unroll
  for (int g = 0; g < DK_MAXG; ++g) {
    if (g >= G) break;
    const float s = live ? acc[g] : -INFINITY;
    p.S[((int64_t)b * p.Hq + hk * G + g) * ks + k] = s;
    float m = s;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5][g] = m;
  }
  __syncthreads();
  if (threadIdx.x < G) {
    float m = -INFINITY;
    for (int w = 0; w < DK_KEYS / 32; ++w) m = fmaxf(m, red[w][threadIdx.x]);
    p.pmax[((int64_t)b * p.Hq + hk * G + threadIdx.x) * p.nsplit + split] = m;
  }
}

// e = exp2((S - m) log2 e) for one key of every head of the group, the NVFP4
// fake-quant of e per 16 keys (16 consecutive threads hold one block), then
// O-partial = P-hat V-hat over the split's keys.
__global__ void __launch_bounds__(DK_KEYS) decode_pv_kernel(DecodeArgs p) {
  const int split = blockIdx.x, bk = blockIdx.y;
  const int b = bk / p.Hkv, hk = bk % p.Hkv;
  const int G = p.Hq / p.Hkv;
  __shared__ float ph[DK_MAXG][DK_KEYS];  // P-hat
  __shared__ float lred[DK_KEYS / 32][DK_MAXG];
  __shared__ float opart[2][DK_MAXG][DK_D];
  const int ks = p.nsplit * DK_KEYS;
  const int k = split * DK_KEYS + threadIdx.x;
  const float log2e = 1.4426950408889634f, r6 = __frcp_rn(6.0f);
  for (int g = 0; g < G; ++g) {
    const int h = hk * G + g;
    float m = -INFINITY;
    for (int s = 0; s < p.nsplit; ++s) m = fmaxf(m, p.pmax[((int64_t)b * p.Hq + h) * p.nsplit + s]);
    const float sv = p.S[((int64_t)b * p.Hq + h) * ks + k];
    const float e = (k < p.len && m != -INFINITY) ? exp2f(__fmul_rn(sv - m, log2e)) : 0.0f;
    // block of 16 keys = 16 consecutive lanes
    float am = e;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const uint8_t sb = e4m3_satfinite(__fmul_rn(am, r6));
    const float s = e4m3_to_f32(sb);
    const float rs = s == 0.0f ? 0.0f : __frcp_rn(s);
    const uint32_t byte = e2m1x2(__fmaf_rn(e, rs, 0.0f), 0.0f);
    ph[g][threadIdx.x] = __fmul_rn(e2m1_value(byte & 15u), s);
    float l = e;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if ((threadIdx.x & 31) == 0) lred[threadIdx.x >> 5][g] = l;
  }
  __syncthreads();
  if (threadIdx.x < G) {
    float l = 0.0f;
    for (int w = 0; w < DK_KEYS / 32; ++w) l += lred[w][threadIdx.x];
    p.lpart[((int64_t)b * p.Hq + hk * G + threadIdx.x) * p.nsplit + split] = l;
  }
  // O-partial: thread (half, d) sums keys of its parity
  const int d = threadIdx.x % DK_D, half = threadIdx.x / DK_D;
  float o[DK_MAXG];
#pragma unroll
  for (int g = 0; g < DK_MAXG; ++g) o[g] = 0.0f;
  const int kend = min(DK_KEYS, p.len - split * DK_KEYS);
  for (int kk = half; kk < kend; kk += 2) {
    const int key = split * DK_KEYS + kk;
    const int64_t row = ((int64_t)b * p.Hkv + hk) * p.Tmax + key;
    const uint8_t cb = p.v_codes[row * (DK_D / 2) + d / 2];
    const float code = e2m1_value((d & 1) ? (cb >> 4) : (cb & 15u));
    const float v = __fmul_rn(__fmul_rn(code, e4m3_to_f32(p.v_scales[row * DK_D + d])),
                              p.v_g[(int64_t)b * p.Tmax + key]);
#pragma unroll
    for (int g = 0; g < DK_MAXG; ++g)
      if (g < G) o[g] = __fmaf_rn(ph[g][kk], v, o[g]);
  }
#pragma unroll
  for (int g = 0; g < DK_MAXG; ++g)
    if (g < G) opart[half][g][d] = o[g];
  __syncthreads();
  for (int i = threadIdx.x; i < G * DK_D; i += DK_KEYS) {
    const int g = i / DK_D, dd = i % DK_D;
    p.opart[(((int64_t)b * p.Hq + hk * G + g) * p.nsplit + split) * DK_D + dd] = opart[0][g][dd] + opart[1][g][dd];
  }
}

__global__ void __launch_bounds__(DK_D) decode_combine_kernel(DecodeArgs p) {
  const int bh = blockIdx.x, d = threadIdx.x;
  float o = 0.0f, l = 0.0f;
  for (int s = 0; s < p.nsplit; ++s) {
    o += p.opart[((int64_t)bh * p.nsplit + s) * DK_D + d];
    l += p.lpart[(int64_t)bh * p.nsplit + s];
  }
  p.out[(int64_t)bh * DK_D + d] = o / l;
}

}  // namespace
}  // namespace fp4

using namespace fp4;

extern "C" int64_t fp4attn_decode_workspace_size(int B, int Hq, int len) {
  if (B <= 0 || Hq <= 0 || len <= 0) return -1;
  const int64_t nsplit = (len + DK_KEYS - 1) / DK_KEYS;
  const int64_t bh = (int64_t)B * Hq;
  return (bh * nsplit * DK_KEYS + bh * nsplit * (DK_D + 2)) * (int64_t)sizeof(float);
}

extern "C" int fp4attn_decode(const float* qhat, const uint8_t* k_codes, const uint8_t* k_scales, const float* k_g,
                              const uint8_t* v_codes, const uint8_t* v_scales, const float* v_g, int B, int Hq,
                              int Hkv, int D, int len, int Tmax, float scaling, float* out, void* workspace,
                              int64_t workspace_bytes, void* stream) {
  clear_error();
  if (!qhat || !k_codes || !k_scales || !k_g || !v_codes || !v_scales || !v_g || !out || !workspace)
    return set_error(FP4ATTN_ERR_ARG, "null pointer");
  if (D != DK_D) return set_error(FP4ATTN_ERR_UNSUPPORTED, "head_dim must be %d", DK_D);
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || len <= 0 || Tmax < len)
    return set_error(FP4ATTN_ERR_ARG, "bad shape");
  if (Hq / Hkv > DK_MAXG) return set_error(FP4ATTN_ERR_UNSUPPORTED, "more than %d query heads per KV head", DK_MAXG);
  if (((uintptr_t)k_codes | (uintptr_t)v_codes) % 16 || (uintptr_t)k_scales % 8)
    return set_error(FP4ATTN_ERR_ARG, "cache buffers must be 16-byte (codes) / 8-byte (K scales) aligned");
  const int64_t need = fp4attn_decode_workspace_size(B, Hq, len);
  if (workspace_bytes < need) return set_error(FP4ATTN_ERR_ARG, "workspace of %lld bytes, %lld needed",
                                               (long long)workspace_bytes, (long long)need);
  const int nsplit = (len + DK_KEYS - 1) / DK_KEYS;
  const int64_t bh = (int64_t)B * Hq;
  float* ws = static_cast<float*>(workspace);
  DecodeArgs a{qhat, k_codes, k_scales, k_g, v_codes, v_scales, v_g, B, Hq, Hkv, len, Tmax, nsplit, scaling,
               ws, ws + bh * nsplit * DK_KEYS, ws + bh * nsplit * (DK_KEYS + 1),
               ws + bh * nsplit * (DK_KEYS + 1 + DK_D), out};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid(nsplit, B * Hkv);
  decode_scores_kernel<<<grid, DK_KEYS, 0, st>>>(a);
  if (int e = check_launch("decode_scores_kernel")) return e;
  decode_pv_kernel<<<grid, DK_KEYS, 0, st>>>(a);
  if (int e = check_launch("decode_pv_kernel")) return e;
  decode_combine_kernel<<<(unsigned)bh, DK_D, 0, st>>>(a);
  return check_launch("decode_combine_kernel");
}
