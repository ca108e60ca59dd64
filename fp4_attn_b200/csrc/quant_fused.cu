// quant_fused.cu -- single-pass NVFP4 quantize for the per-tensor global
// scale (fp4q_quantize gmode 3) when the whole tensor fits in the shared
// memory of the GPU's SMs.
//
// The per-tensor scale g = max|x| * recip(global_sf_max) is needed before any
// block is quantized, so a plain implementation reads the tensor twice
// (max pre-pass, then quantize).  Here one cooperative launch with one CTA per
// SM copies its contiguous slice of the tensor into shared memory (bulk
// copies), reduces its maximum, meets the other CTAs at a grid-wide barrier,
// and quantizes from shared memory: the tensor crosses HBM once.  Same
// arithmetic, op for op, as quant_rows_kernel in fp32 (quant_block): x * rg,
// block max, E4M3 scale by the torch cast, x * recip(s) + 0, E2M1 RNE.
//
// The barrier words live in the first 12 bytes of the codes output (zeroed by
// the host before the launch): [0] bits of the running max, [1] arrivals,
// [2] departures.  CTA 0 writes the codes of blocks 0 and 1 (those bytes) and
// g last, once every CTA has read the max.  Every wait is bounded.
#include <stdint.h>

#include <algorithm>

#include "quant_impl.cuh"
#include "sm100.cuh"

namespace fp4 {

FP4_DEFINE_STATUS_READER(quant_status)

namespace {

constexpr int QF_THREADS = 1024;
constexpr int QF_PIECES = 8;  // bulk copies per slice, each with its own barrier (the max runs as they land)
constexpr int QF_SMEM_MAX = 232448 - 1024;  // dynamic shared memory for the slice (sm_100 limit minus headroom)

struct QFArgs {
  const void* x;
  int64_t nelem;  // multiple of 16
  int64_t chunk;  // elements per CTA, multiple of 16
  uint8_t* codes;
  uint8_t* scales;
  float* g;
  float gsf_max;
};

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* w) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(w) : "memory");
  return v;
}
// Every memory operation of this thread before it is visible before the increment.
__device__ __forceinline__ void add_release(unsigned int* w, unsigned int v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(w), "r"(v) : "memory");
}

// Bounded spin until *w >= target (acquire loads: what the arriving threads
// wrote before their release is visible afterwards); false after 2 s.
__device__ bool wait_count(const unsigned int* w, unsigned int target, unsigned int site) {
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 0;; ++i) {
    if (ld_acquire(w) >= target) return true;
    if ((i & 63) == 63) {
      if (dev_failed()) return false;
      if (globaltimer() - t0 > kWaitNs) {
        dev_fail(site);
        return false;
      }
    }
  }
}

// Per 16-bit lane: max(|a|, |b|) in the input type, NaN winning (max.NaN), exact.
template <int DT>
__device__ __forceinline__ uint32_t absmax_x2(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (DT == FP4_DT_BF16)
    asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a & 0x7FFF7FFFu), "r"(b & 0x7FFF7FFFu));
  else
    asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a & 0x7FFF7FFFu), "r"(b & 0x7FFF7FFFu));
  return r;
}

template <int DT>
__global__ void __launch_bounds__(QF_THREADS, 1) quant_tensor_fused_kernel(QFArgs p) {
  using T = typename In<DT>::T;
  constexpr int A = FP4_ARITH_F32;
  extern __shared__ __align__(128) uint8_t qf_slice[];
  __shared__ __align__(8) uint64_t bar[QF_PIECES];
  __shared__ float wmax[QF_THREADS / 32];
  __shared__ float rcp_tab[128];
  __shared__ float s_g, s_rg;
  __shared__ int s_ok;
  __shared__ uint32_t stash[4];  // CTA 0: codes words of blocks 0 and 1, written last
  unsigned int* cw = reinterpret_cast<unsigned int*>(p.codes);
  const unsigned int G = gridDim.x;
  const int64_t e0 = (int64_t)blockIdx.x * p.chunk;
  const int64_t e1 = e0 + p.chunk < p.nelem ? e0 + p.chunk : p.nelem;
  const int64_t cnt = e1 > e0 ? e1 - e0 : 0;
  const uint32_t bytes = (uint32_t)(cnt * (int64_t)sizeof(T));
  if (threadIdx.x < 128) rcp_tab[threadIdx.x] = recip<A>(e4m3_to_f32((uint8_t)threadIdx.x));
  // the slice in QF_PIECES pieces of whole 16-byte vectors (the last one takes the rest)
  const int nv = (int)(bytes / 16);
  const int pv = (nv + QF_PIECES - 1) / QF_PIECES;
  if (threadIdx.x == 0) {
    for (int k = 0; k < QF_PIECES; ++k) mbar_init(&bar[k], 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(p.x) + e0 * (int64_t)sizeof(T);
    for (int k = 0; k < QF_PIECES; ++k) {
      const int v0 = k * pv, v1 = v0 + pv < nv ? v0 + pv : nv;
      if (v1 > v0) {
        const uint32_t pb = (uint32_t)(v1 - v0) * 16u;
        mbar_arrive_expect_tx(&bar[k], pb);
        bulk_load(qf_slice + (size_t)v0 * 16, src + (size_t)v0 * 16, pb, &bar[k]);
      } else {
        mbar_arrive(&bar[k]);
      }
    }
  }
  // ---- maximum of |x| over the slice (torch.max semantics: NaN wins), piece by piece as it lands.
  // 16-bit inputs: on packed pairs in the input type (|x| by clearing the sign bits, exact), widened once at the end.
  float m = 0.0f;
  uint32_t m2 = 0u;
  const uint4* s4 = reinterpret_cast<const uint4*>(qf_slice);
  bool loaded = true;
  for (int k = 0; k < QF_PIECES; ++k) {
    loaded = mbar_wait(&bar[k], 0, 0x301) && loaded;
    if (!loaded) break;
    const int v1 = (k + 1) * pv < nv ? (k + 1) * pv : nv;
    for (int i = k * pv + threadIdx.x; i < v1; i += QF_THREADS) {
      const uint4 u = s4[i];
      if constexpr (sizeof(T) == 2) {
        m2 = absmax_x2<DT>(m2, absmax_x2<DT>(absmax_x2<DT>(u.x, u.y), absmax_x2<DT>(u.z, u.w)));
      } else {
        const float* e = reinterpret_cast<const float*>(&u);
        m = nanmax(m, nanmax(absmax3(e[0], e[1], e[2]), fabsf(e[3])));
      }
    }
  }
  if constexpr (sizeof(T) == 2) {
    const T* h = reinterpret_cast<const T*>(&m2);
    m = nanmax(In<DT>::f(h[0]), In<DT>::f(h[1]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = nanmax(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
#pragma unroll
    for (int w = 1; w < QF_THREADS / 32; ++w) m = nanmax(m, wmax[w]);
    atomicMax(&cw[0], __float_as_uint(m));
    add_release(&cw[1], 1u);  // arrival, after the max
    bool ok = loaded && wait_count(&cw[1], G, 0x302);
    const float mx = __uint_as_float(ld_acquire(&cw[0]));
    const float g = mul<A>(mx, recip<A>(rnd<A>(p.gsf_max)));  // fp4_quant_utils.py:139
    s_g = g;
    s_rg = recip<A>(g);
    add_release(&cw[2], 1u);  // departure, after reading the max
    s_ok = ok ? 1 : 0;
  }
  __syncthreads();
  if (!s_ok) return;
  // ---- quantize from shared memory: lanes 2i and 2i+1 hold the two halves of a block;
  // each thread takes two halves per step (independent chains the scheduler interleaves)
  const float rg = s_rg, r6 = recip6<A>();
  const int64_t b0 = e0 / 16;  // first block of the slice
  const int nhalf = (int)(cnt / 8);
  const float2 rg2 = make_float2(rg, rg), zero2 = make_float2(0.0f, 0.0f);
  for (int base = 0; base < nhalf; base += 2 * QF_THREADS) {
    float2 v[2][4];  // (x, x') pairs of a half block, kept as register pairs for the f32x2 ops
    float am[2];
    bool live[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int hidx = base + u * QF_THREADS + (int)threadIdx.x;
      live[u] = hidx < nhalf;
      if (live[u]) {
        if constexpr (sizeof(T) == 4) {
          const uint4 u0 = s4[2 * hidx], u1 = s4[2 * hidx + 1];
          v[u][0] = make_float2(__uint_as_float(u0.x), __uint_as_float(u0.y));
          v[u][1] = make_float2(__uint_as_float(u0.z), __uint_as_float(u0.w));
          v[u][2] = make_float2(__uint_as_float(u1.x), __uint_as_float(u1.y));
          v[u][3] = make_float2(__uint_as_float(u1.z), __uint_as_float(u1.w));
        } else {
          const uint4 q = s4[hidx];
          const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
          for (int k = 0; k < 4; ++k) v[u][k] = make_float2(In<DT>::f(e[2 * k]), In<DT>::f(e[2 * k + 1]));
        }
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) v[u][k] = zero2;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) v[u][k] = __fmul2_rn(v[u][k], rg2);  // x * recip(g)
      float a = absmax3(v[u][0].x, v[u][0].y, v[u][1].x);
      a = absmax3(a, v[u][1].y, v[u][2].x);
      a = absmax3(a, v[u][2].y, v[u][3].x);
      am[u] = nanmax(a, fabsf(v[u][3].y));
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) am[u] = nanmax(am[u], __shfl_xor_sync(0xffffffffu, am[u], 1));  // the block's other half
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int hidx = base + u * QF_THREADS + (int)threadIdx.x;
      const uint8_t sb = e4m3_torch(mul<A>(am[u], r6));
      const float rs = rcp_tab[sb & 0x7F];
      const bool nan_block = (sb & 0x7F) == 0x7F;
      const float2 rs2 = make_float2(rs, rs);
      float q[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        // x * recip(s) + 0: one rounding of the product; + 0 turns -0.0 into +0.0 (torch.sign(-0.0) == 0)
        const float2 t = __ffma2_rn(v[u][k], rs2, zero2);
        q[2 * k] = t.x;
        q[2 * k + 1] = t.y;
      }
      const uint32_t word = nan_block ? 0u : e2m1x8(q);
      if (live[u]) {
        const int64_t blk = b0 + (hidx >> 1);
        if (blk < 2) {  // only in CTA 0 (its slice starts at block 0 and holds at least 2 blocks)
          stash[hidx] = word;  // bytes 0..15 of codes hold the barrier words until the end
        } else {
          reinterpret_cast<uint32_t*>(p.codes)[2 * blk + (hidx & 1)] = word;
        }
        if ((hidx & 1) == 0) p.scales[blk] = sb;
      }
    }
  }
  if (blockIdx.x == 0) {
    __syncthreads();
    if (threadIdx.x == 0) {
      // every CTA has read the max: the barrier words can become codes
      if (wait_count(&cw[2], G, 0x303)) {
        const int nst = (int)std::min<int64_t>(4, nhalf);
        for (int i = 0; i < nst; ++i) reinterpret_cast<uint32_t*>(p.codes)[i] = stash[i];
        p.g[0] = s_g;
      }
    }
  }
}

}  // namespace

// Single-pass per-tensor quantize of a contiguous tensor whose elements are a
// multiple of 16 (codes/scales contiguous, linear scale layout, fp32
// arithmetic).  Returns -1 when the tensor does not fit on chip or the device
// cannot run the cooperative launch (the caller then runs the two-pass path).
int quant_tensor_fused(const void* x, int in_dtype, int64_t nelem, uint8_t* codes, uint8_t* scales, float* g,
                       float gsf_max, cudaStream_t st) {
  const int esz = in_dtype == FP4_DT_F32 ? 4 : 2;
  int dev = 0, sms = 0, coop = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
  if (!coop || sms <= 0 || nelem < 32 || nelem % 16) return -1;
  // at least two blocks per CTA, so CTA 0 owns blocks 0 and 1 (the barrier words)
  const int64_t chunk = std::max<int64_t>(32, (nelem / 16 + sms - 1) / sms * 16);
  const int64_t smem = chunk * esz;
  if (smem > QF_SMEM_MAX || smem % 16) return -1;
  const int grid = (int)((nelem + chunk - 1) / chunk);
  void* fn = nullptr;
  switch (in_dtype) {
    case FP4_DT_F32: fn = (void*)quant_tensor_fused_kernel<FP4_DT_F32>; break;
    case FP4_DT_BF16: fn = (void*)quant_tensor_fused_kernel<FP4_DT_BF16>; break;
    case FP4_DT_F16: fn = (void*)quant_tensor_fused_kernel<FP4_DT_F16>; break;
    default: return -1;
  }
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, QF_THREADS, (size_t)smem) != cudaSuccess ||
      per_sm < 1 || grid > per_sm * sms) {
    cudaGetLastError();
    return -1;
  }
  if (cudaMemsetAsync(codes, 0, 12, st) != cudaSuccess) return set_error(FP4ATTN_ERR_CUDA, "memset");
  QFArgs a{x, nelem, chunk, codes, scales, g, gsf_max};
  void* args[] = {&a};
  if (cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(QF_THREADS), args, (size_t)smem, st) != cudaSuccess)
    return check_launch("quant_tensor_fused_kernel");
  return check_launch("quant_tensor_fused_kernel");
}

}  // namespace fp4
