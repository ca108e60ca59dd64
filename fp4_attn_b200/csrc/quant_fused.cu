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
constexpr int QF_PIECES = 4;  // bulk copies per slice, each with its own barrier
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

// Bounded spin until *w >= target (volatile reads); false after 2 s.
__device__ bool wait_count(const unsigned int* w, unsigned int target, unsigned int site) {
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 0;; ++i) {
    if (*reinterpret_cast<const volatile unsigned int*>(w) >= target) return true;
    if ((i & 63) == 63) {
      if (dev_failed()) return false;
      if (globaltimer() - t0 > kWaitNs) {
        dev_fail(site);
        return false;
      }
      __nanosleep(64);
    }
  }
}

template <int DT>
__global__ void __launch_bounds__(QF_THREADS, 1) quant_tensor_fused_kernel(QFArgs p) {
  using T = typename In<DT>::T;
  constexpr int A = FP4_ARITH_F32;
  constexpr int PER = 16 / (int)sizeof(T);  // elements per 16-byte vector
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
  // ---- maximum of |x| over the slice (torch.max semantics: NaN wins), piece by piece as it lands
  float m = 0.0f;
  const uint4* s4 = reinterpret_cast<const uint4*>(qf_slice);
  bool loaded = true;
  for (int k = 0; k < QF_PIECES; ++k) {
    loaded = mbar_wait(&bar[k], 0, 0x301) && loaded;
    if (!loaded) break;
    const int v1 = (k + 1) * pv < nv ? (k + 1) * pv : nv;
    for (int i = k * pv + threadIdx.x; i < v1; i += QF_THREADS) {
      const uint4 u = s4[i];
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < PER; ++j) m = nanmax(m, fabsf(rnd<A>(In<DT>::f(e[j]))));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = nanmax(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
#pragma unroll
    for (int w = 1; w < QF_THREADS / 32; ++w) m = nanmax(m, wmax[w]);
    atomicMax(&cw[0], __float_as_uint(m));
    __threadfence();
    atomicAdd(&cw[1], 1u);
    bool ok = loaded && wait_count(&cw[1], G, 0x302);
    __threadfence();
    const float mx = __uint_as_float(*reinterpret_cast<const volatile unsigned int*>(&cw[0]));
    const float g = mul<A>(mx, recip<A>(rnd<A>(p.gsf_max)));  // fp4_quant_utils.py:139
    s_g = g;
    s_rg = recip<A>(g);
    __threadfence();
    atomicAdd(&cw[2], 1u);
    s_ok = ok ? 1 : 0;
  }
  __syncthreads();
  if (!s_ok) return;
  // ---- quantize from shared memory: lanes 2i and 2i+1 hold the two halves of a block
  const float rg = s_rg, r6 = recip<A>(6.0f);
  const int64_t b0 = e0 / 16;  // first block of the slice
  const int nhalf = (int)(cnt / 8);
  for (int base = 0; base < nhalf; base += QF_THREADS) {
    const int hidx = base + (int)threadIdx.x;
    const bool live = hidx < nhalf;
    float v[8];
    if (live) {
      if constexpr (sizeof(T) == 4) {
        const uint4 u0 = s4[2 * hidx], u1 = s4[2 * hidx + 1];
        const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = rnd<A>(__uint_as_float(w[k]));
      } else {
        const uint4 u = s4[hidx];
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = rnd<A>(In<DT>::f(e[k]));
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = 0.0f;
    }
#pragma unroll
    for (int k = 0; k < 8; k += 2) mul2(v[k], v[k + 1], rg);
    float am = absmax3(v[0], v[1], v[2]);
    am = absmax3(am, v[3], v[4]);
    am = absmax3(am, v[5], v[6]);
    am = nanmax(am, fabsf(v[7]));
    am = nanmax(am, __shfl_xor_sync(0xffffffffu, am, 1));  // the block's other half
    if (!live) continue;
    const uint8_t sb = e4m3_torch(mul<A>(am, r6));
    const float rs = rcp_tab[sb & 0x7F];
    const bool nan_block = (sb & 0x7F) == 0x7F;
#pragma unroll
    for (int k = 0; k < 8; k += 2) mulz2(v[k], v[k + 1], rs);
    const uint32_t word = nan_block ? 0u : e2m1x8(v);
    const int64_t blk = b0 + (hidx >> 1);
    if (blk < 2) {  // only in CTA 0 (its slice starts at block 0 and holds at least 2 blocks)
      stash[hidx] = word;  // bytes 0..15 of codes hold the barrier words until the end
    } else {
      reinterpret_cast<uint32_t*>(p.codes)[2 * blk + (hidx & 1)] = word;
    }
    if ((hidx & 1) == 0) p.scales[blk] = sb;
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
