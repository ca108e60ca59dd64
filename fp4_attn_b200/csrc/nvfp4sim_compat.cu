// nvfp4sim_compat.cu -- the five functions of the reference extension module
// `nvfp4sim` (fast_fp4/wrapper.cpp:40-46), re-implemented for sm_100a with the
// reference's numerics (fast_fp4/nvfp4sim.cu):
//   * amax with a 1e-10 floor, fmaxf (NaN inputs ignored)          (:104-113)
//   * scale byte = satfinite E4M3 of (double)amax * (1.0/6.0)      (:116)
//   * search: the 16 candidate bytes base + c - 7 (8-bit wrap)     (:117)
//   * inv = (float)(1.0 / (double)scale)                            (:119)
//   * E2M1 encode rounds half away from zero through a denormal
//     bit trick (:76-85); decode is its inverse (:87-94)
//   * winner = smallest loss with its low 4 bits replaced by the
//     candidate index; a group whose every loss is NaN is left unwritten
//     (:134-153)
// The loss is summed without FMA contraction (explicit _rn intrinsics).
//
// Work split: CANDS consecutive threads evaluate the candidates of one group
// of 16 (CANDS = 16 with search, 1 without); each thread reads the group with
// 16-byte loads, and the candidates meet in a shuffle min-reduction.
#include "common.cuh"
#include "status.h"

namespace fp4 {

__device__ __forceinline__ uint32_t ref_f32_to_f4(float a) {
  const float kScale = 1.1754943508222875e-38f;  // 2^-126
  a = __fmul_rn(fminf(fmaxf(-6.0f, a), 6.0f), kScale);
  uint32_t u = __float_as_uint(a) + (1u << 21);
  return ((u >> 22) & 7u) | ((u >> 28) & 8u);
}

__device__ __forceinline__ float ref_f4_to_f32(uint32_t c) {
  const float kIScale = 8.507059173023462e+37f;  // 2^126
  return __fmul_rn(__uint_as_float(((c & 7u) << 22) | ((c & 8u) << 28)), kIScale);
}

template <typename T>
__device__ __forceinline__ void load16(float x[16], const T* p);

template <>
__device__ __forceinline__ void load16<float>(float x[16], const float* p) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float4 f = __ldg(q + j);
    x[4 * j] = f.x;
    x[4 * j + 1] = f.y;
    x[4 * j + 2] = f.z;
    x[4 * j + 3] = f.w;
  }
}

template <>
__device__ __forceinline__ void load16<__half>(float x[16], const __half* p) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    uint4 u = __ldg(q + j);
    const __half* h = reinterpret_cast<const __half*>(&u);
#pragma unroll
    for (int k = 0; k < 8; ++k) x[8 * j + k] = __half2float(h[k]);
  }
}

template <typename T, int CANDS>
__global__ void __launch_bounds__(256) to_nvf4_kernel(uint64_t* xq, uint8_t* xs, const T* x, int64_t ngroups) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t grp = tid / CANDS;
  const int cand = (int)(tid % CANDS);
  const bool live = grp < ngroups;
  float v[16];
  if (live) {
    load16<T>(v, x + grp * 16);
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = 0.0f;
  }
  float amax = 1e-10f;
#pragma unroll
  for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));
  const uint8_t base = e4m3_satfinite((float)((double)amax * (1.0 / 6.0)));
  const uint8_t sb = CANDS > 1 ? (uint8_t)(base + (cand - 7)) : base;
  const float sc = e4m3_to_f32(sb);
  const float inv = (float)(1.0 / (double)sc);
  float loss = 0.0f;
  uint64_t q = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t lo = ref_f32_to_f4(__fmul_rn(v[2 * i], inv));
    const uint32_t hi = ref_f32_to_f4(__fmul_rn(v[2 * i + 1], inv));
    q |= (uint64_t)(lo | (hi << 4)) << (8 * i);
    const float d0 = __fsub_rn(__fmul_rn(ref_f4_to_f32(lo), sc), v[2 * i]);
    const float d1 = __fsub_rn(__fmul_rn(ref_f4_to_f32(hi), sc), v[2 * i + 1]);
    loss = __fadd_rn(loss, __fmul_rn(d0, d0));
    loss = __fadd_rn(loss, __fmul_rn(d1, d1));
  }
  const float tagged = __uint_as_float((__float_as_uint(loss) & ~15u) | (uint32_t)cand);
  float best = tagged;
#pragma unroll
  for (int o = CANDS / 2; o > 0; o >>= 1) best = fminf(best, __shfl_xor_sync(0xffffffffu, best, o));
  if (live && tagged == best) {
    xq[grp] = q;
    xs[grp] = sb;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) from_nvf4_kernel(T* out, const uint64_t* xq, const uint8_t* xs, int64_t ngroups) {
  const int64_t grp = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (grp >= ngroups) return;
  const uint64_t q = xq[grp];
  const float sc = e4m3_to_f32(xs[grp]);
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __fmul_rn(ref_f4_to_f32((uint32_t)(q >> (4 * i)) & 15u), sc);
  if constexpr (sizeof(T) == 4) {
    float4* o = reinterpret_cast<float4*>(out + grp * 16);
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
    uint4 u[2];
    __half* h = reinterpret_cast<__half*>(u);
#pragma unroll
    for (int i = 0; i < 16; ++i) h[i] = __float2half_rn(v[i]);
    uint4* o = reinterpret_cast<uint4*>(out + grp * 16);
    o[0] = u[0];
    o[1] = u[1];
  }
}

static int check_groups(int64_t ngroups, const void* a, const void* b, const void* c) {
  if (ngroups < 0) return set_error(FP4ATTN_ERR_ARG, "negative group count");
  if (ngroups % 2 != 0) return set_error(FP4ATTN_ERR_ARG, "group count must be even (nvfp4sim.cu:175)");
  if (ngroups > 0 && (!a || !b || !c)) return set_error(FP4ATTN_ERR_ARG, "null pointer");
  if ((uintptr_t)c % 16 != 0 || (uintptr_t)a % 8 != 0) return set_error(FP4ATTN_ERR_ARG, "misaligned buffer");
  return FP4ATTN_OK;
}

template <typename T, int CANDS>
static int run_to(uint64_t* xq, uint8_t* xs, const T* x, int64_t ngroups, void* stream) {
  clear_error();
  if (int e = check_groups(ngroups, xq, xs, x)) return e;
  if (ngroups == 0) return FP4ATTN_OK;
  const int64_t threads = ngroups * CANDS;
  to_nvf4_kernel<T, CANDS><<<(unsigned)((threads + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      xq, xs, x, ngroups);
  return check_launch("to_nvf4_kernel");
}

template <typename T>
static int run_from(T* out, const uint64_t* xq, const uint8_t* xs, int64_t ngroups, void* stream) {
  clear_error();
  if (int e = check_groups(ngroups, xq, xs, out)) return e;
  if (ngroups == 0) return FP4ATTN_OK;
  from_nvf4_kernel<T><<<(unsigned)((ngroups + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      out, xq, xs, ngroups);
  return check_launch("from_nvf4_kernel");
}

}  // namespace fp4

using namespace fp4;

extern "C" int nvfp4sim_f32_to_nvf4(uint64_t* xq_out, uint8_t* xs_out, const float* x_in, int64_t ngroups, void* stream) {
  return run_to<float, 16>(xq_out, xs_out, x_in, ngroups, stream);
}

extern "C" int nvfp4sim_f32_to_nvf4_nosearch(uint64_t* xq_out, uint8_t* xs_out, const float* x_in, int64_t ngroups,
                                             void* stream) {
  return run_to<float, 1>(xq_out, xs_out, x_in, ngroups, stream);
}

extern "C" int nvfp4sim_f16_to_nvf4(uint64_t* xq_out, uint8_t* xs_out, const uint16_t* x_in, int64_t ngroups,
                                    void* stream) {
  return run_to<__half, 16>(xq_out, xs_out, reinterpret_cast<const __half*>(x_in), ngroups, stream);
}

extern "C" int nvfp4sim_nvf4_to_f32(float* x_out, const uint64_t* xq_in, const uint8_t* xs_in, int64_t ngroups,
                                    void* stream) {
  return run_from<float>(x_out, xq_in, xs_in, ngroups, stream);
}

extern "C" int nvfp4sim_nvf4_to_f16(uint16_t* x_out, const uint64_t* xq_in, const uint8_t* xs_in, int64_t ngroups,
                                    void* stream) {
  return run_from<__half>(reinterpret_cast<__half*>(x_out), xq_in, xs_in, ngroups, stream);
}
