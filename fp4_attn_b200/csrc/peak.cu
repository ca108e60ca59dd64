// peak.cu -- dense NVFP4 tensor-core throughput of this GPU, measured: the
// roofline denominator of the FP4 contractions (attention QK^T, the NVFP4
// GEMM).
//
// One CTA per SM; one elected thread issues back-to-back
// tcgen05.mma.kind::mxf4nvf4.block_scale.block16 instructions (M=128,
// N=128, K=64, the shape the attention kernel issues) from fixed shared-memory
// operands into three TMEM accumulators in rotation, then commits once and
// waits (bounded).  Operands are pseudo-random E2M1 codes with E4M3 scales
// near 1, so the datapath toggles as on real data.  FLOPs per launch =
// ctas * iters * 2 * (2 * 128 * 128 * 64); the caller times the launch with
// CUDA events.  No reference counterpart (a measurement aid).
#include <cuda.h>

#include "fp4attn.h"
#include "sm100.cuh"
#include "status.h"

namespace fp4 {

FP4_DEFINE_STATUS_READER(peak_status)

namespace peak {
constexpr int THREADS = 128;
constexpr int OFF_A = 0, OFF_B = 8192, OFF_SFA = 16384, OFF_SFB = 17408, OFF_BAR = 18432;
constexpr int SMEM_BYTES = OFF_BAR + 64 + 1024;
constexpr uint32_t TMEM_COLS = 512;  // three 128-column accumulators, then the scale atoms
constexpr uint32_t T_SFA = 384, T_SFB = 392;
}  // namespace peak

__device__ __forceinline__ uint32_t peak_hash(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

__global__ void __launch_bounds__(peak::THREADS, 1) mma_peak_kernel(int iters) {
  using namespace peak;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* done = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  const int warp = threadIdx.x / 32;
  // codes: any byte is two valid E2M1 values; scales: E4M3 bytes 0x30..0x3F (0.5 .. 0.94)
  for (int i = threadIdx.x; i < 16384 / 4; i += THREADS)
    reinterpret_cast<uint32_t*>(sm + OFF_A)[i] = peak_hash((uint32_t)i * 2654435761u + blockIdx.x);
  for (int i = threadIdx.x; i < 2048; i += THREADS) sm[OFF_SFA + i] = (uint8_t)(0x30 | (peak_hash(i + 7u) & 0xF));
  if (threadIdx.x == 0) {
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy writes seen by the tensor core
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0 && elect_one_lane()) {
    const uint32_t idq = idesc_nvf4(128, 128);
    tmem_cp_sf_atom(tmem + T_SFA, smem_desc(smem_u32(sm + OFF_SFA), 16, 128, kSwizzleNone));
    tmem_cp_sf_atom(tmem + T_SFA + 4, smem_desc(smem_u32(sm + OFF_SFA + 512), 16, 128, kSwizzleNone));
    tmem_cp_sf_atom(tmem + T_SFB, smem_desc(smem_u32(sm + OFF_SFB), 16, 128, kSwizzleNone));
    tmem_cp_sf_atom(tmem + T_SFB + 4, smem_desc(smem_u32(sm + OFF_SFB + 512), 16, 128, kSwizzleNone));
    for (int i = 0; i < iters; ++i) {
      const uint32_t d = tmem + 128 * (uint32_t)(i % 3);
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const uint64_t ad = smem_desc(smem_u32(sm + OFF_A) + kk * 32, 16, 512, kSwizzle64B);
        const uint64_t bd = smem_desc(smem_u32(sm + OFF_B) + kk * 32, 16, 512, kSwizzle64B);
        mma_nvf4(d, ad, bd, idq, tmem + T_SFA + 4 * kk, tmem + T_SFB + 4 * kk, kk > 0 ? 1u : 0u);
      }
    }
    tc_commit(done);
  }
  __syncwarp();
  if (warp == 0) mbar_wait(done, 0, 0x601);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace fp4

using namespace fp4;

extern "C" int fp4_mma_peak_run(int iters, int num_ctas, void* stream) {
  clear_error();
  if (iters <= 0 || iters > (1 << 20)) return set_error(FP4ATTN_ERR_ARG, "iters must be in [1, 2^20]");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = num_ctas > 0 ? num_ctas : sms;
  if (int e = set_smem_attr((const void*)mma_peak_kernel, peak::SMEM_BYTES)) return e;
  mma_peak_kernel<<<grid, peak::THREADS, peak::SMEM_BYTES, reinterpret_cast<cudaStream_t>(stream)>>>(iters);
  return check_launch("mma_peak_kernel");
}
