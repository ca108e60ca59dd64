// gemm_nvf4.cu -- NVFP4 GEMM on the 5th-generation tensor cores (sm_100a).
//
//   C[m, n] = ga[m] * gb[n] * sum_k (qa[m,k] * sa[m,k/16]) * (qb[n,k] * sb[n,k/16])
//
// with E2M1 codes qa/qb packed two per byte (K-major rows, as fp4q_quantize
// writes them), UE4M3 block scales in the tcgen05 atom layout, and fp32
// global scales per row of A and per row of B (either may be absent = 1).
// This is the contraction behind the attention kernel's S = Q K^T, exposed on
// its own for NVFP4 linear layers.
//
// One CTA per 128x128 output tile.  Warp 0 issues TMA (codes, 128B swizzle)
// and bulk copies (scale atoms) into a 3-stage ring; warp 1 copies the scale
// atoms into TMEM (tcgen05.cp) and issues tcgen05.mma kind::mxf4nvf4
// (K = 64 per instruction, 4 per 256-wide stage) into a 128-column fp32 TMEM
// accumulator; warps 2-5 drain TMEM, apply the global scales and store.
#include <cuda.h>

#include "common.cuh"
#include "sm100.cuh"
#include "status.h"
#include "tmap.h"

namespace fp4 {

namespace gemm {
constexpr int BM = 128, BN = 128, BK = 256;  // BK in elements (128 bytes of codes per row)
constexpr int STAGES = 3;  // 109 KB of ring: two CTAs per SM, so one's epilogue overlaps the other's main loop
constexpr int A_BYTES = BM * BK / 2, B_BYTES = BN * BK / 2;
constexpr int SF_BYTES = 4 * 512;  // 4 atoms of 128 rows x 4 scales
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + 2 * SF_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 256;  // 128 accumulator + STAGES * (16 SFA + 16 SFB)
}  // namespace gemm

struct GemmArgs {
  const uint8_t* sfa;  // tcgen05 atoms, nkb4 groups per 128-row block
  const uint8_t* sfb;
  const float* ga;  // [M] or null
  const float* gb;  // [N] or null
  float* c;
  int M, N, K;
  int64_t ldc;
  int nkb4;  // K / 64
};

__global__ void __launch_bounds__(gemm::THREADS, 2)
    gemm_nvf4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs p) {
  using namespace gemm;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  // set by the MMA thread when a wait gave up: the accumulator is then partial and the
  // epilogue stores nothing (the done commit is still issued, so no MMA is in flight
  // when TMEM is released)
  volatile uint32_t* mma_failed = tmem_slot + 1;

  const int warp = threadIdx.x / 32;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int ksteps = p.K / BK;

  if (threadIdx.x == 0) {
    *mma_failed = 0u;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t acc = tmem;  // columns [0, 128)

  if (warp == 0 && elect_one_lane()) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int k = 0; k < ksteps; ++k) {
      const int s = k % STAGES;
      if (k >= STAGES && !mbar_wait(&empty[s], ((k / STAGES) - 1) & 1, 0x101)) break;
      uint8_t* st = smem + s * STAGE_BYTES;
      mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
      tma_load_2d(st, &tmA, &full[s], k * (BK / 2), m0);
      tma_load_2d(st + A_BYTES, &tmB, &full[s], k * (BK / 2), n0);
      bulk_load(st + A_BYTES + B_BYTES, p.sfa + ((int64_t)(m0 / 128) * p.nkb4 + k * 4) * 512, SF_BYTES, &full[s]);
      bulk_load(st + A_BYTES + B_BYTES + SF_BYTES, p.sfb + ((int64_t)(n0 / 128) * p.nkb4 + k * 4) * 512, SF_BYTES,
                &full[s]);
    }
  } else if (warp == 1 && elect_one_lane()) {
    const uint32_t idesc = idesc_nvf4(BM, BN);
    bool ok = true;
    for (int k = 0; k < ksteps && ok; ++k) {
      const int s = k % STAGES;
      if (!mbar_wait(&full[s], (k / STAGES) & 1, 0x102)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint8_t* st = smem + s * STAGE_BYTES;
      const uint32_t sfa_t = tmem + 128 + s * 32, sfb_t = sfa_t + 16;
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        tmem_cp_sf_atom(sfa_t + 4 * a, smem_desc(smem_u32(st + A_BYTES + B_BYTES + a * 512), 16, 128, kSwizzleNone));
        tmem_cp_sf_atom(sfb_t + 4 * a,
                        smem_desc(smem_u32(st + A_BYTES + B_BYTES + SF_BYTES + a * 512), 16, 128, kSwizzleNone));
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t ad = smem_desc(smem_u32(st) + kk * 32, 16, 1024, kSwizzle128B);
        const uint64_t bd = smem_desc(smem_u32(st + A_BYTES) + kk * 32, 16, 1024, kSwizzle128B);
        mma_nvf4(acc, ad, bd, idesc, sfa_t + 4 * kk, sfb_t + 4 * kk, (k > 0 || kk > 0) ? 1u : 0u);
      }
      tc_commit(&empty[s]);
    }
    if (!ok) {
      *mma_failed = 1u;
      __threadfence_block();
    }
    tc_commit(done);
  } else if (warp >= 2) {
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + (threadIdx.x & 31);
    const bool ok = mbar_wait(done, 0, 0x103) && *mma_failed == 0u;
    tc_fence_after();
    if (ok) {
      const int m = m0 + row;
      const float ga = (p.ga && m < p.M) ? p.ga[m] : 1.0f;
      const bool vec_out = p.ldc % 4 == 0 && (uintptr_t)p.c % 16 == 0 && (uintptr_t)p.gb % 16 == 0;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(acc + ((uint32_t)(quarter * 32) << 16) + c, r);
        tmem_ld_wait();
        if (m < p.M) {
          float* dst = p.c + (int64_t)m * p.ldc + n0 + c;
          if (vec_out && n0 + c + 32 <= p.N) {
            // 16-byte stores of the row's 32 columns (same products, same order)
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const float4 gb = p.gb ? *reinterpret_cast<const float4*>(p.gb + n0 + c + j)
                                     : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
              float4 o;
              o.x = __uint_as_float(r[j]) * ga * gb.x;
              o.y = __uint_as_float(r[j + 1]) * ga * gb.y;
              o.z = __uint_as_float(r[j + 2]) * ga * gb.z;
              o.w = __uint_as_float(r[j + 3]) * ga * gb.w;
              *reinterpret_cast<float4*>(dst + j) = o;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int n = n0 + c + j;
              if (n < p.N) {
                const float gb = p.gb ? p.gb[n] : 1.0f;
                dst[j] = __uint_as_float(r[j]) * ga * gb;
              }
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

FP4_DEFINE_STATUS_READER(gemm_status)

static int make_codes_map(CUtensorMap* map, const uint8_t* codes, int rows, int K, int64_t ld_bytes) {
  return encode_tiled_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, codes, (uint64_t)(K / 2), (uint64_t)rows,
                         (uint64_t)ld_bytes, gemm::BK / 2, 128, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace fp4

using namespace fp4;

extern "C" int fp4_gemm_nvf4(const uint8_t* a_codes, const uint8_t* a_scales, const float* a_g, const uint8_t* b_codes,
                             const uint8_t* b_scales, const float* b_g, float* c, int M, int N, int K, int64_t lda,
                             int64_t ldb, int64_t ldc, void* stream) {
  clear_error();
  if (M <= 0 || N <= 0 || K <= 0) return set_error(FP4ATTN_ERR_ARG, "bad shape");
  if (K % gemm::BK != 0) return set_error(FP4ATTN_ERR_UNSUPPORTED, "K must be a multiple of %d", gemm::BK);
  if (!a_codes || !b_codes || !a_scales || !b_scales || !c) return set_error(FP4ATTN_ERR_ARG, "null pointer");
  if (lda % 16 || ldb % 16 || (uintptr_t)a_codes % 16 || (uintptr_t)b_codes % 16)
    return set_error(FP4ATTN_ERR_ARG, "code rows must be 16-byte aligned");
  if ((uintptr_t)a_scales % 16 || (uintptr_t)b_scales % 16) return set_error(FP4ATTN_ERR_ARG, "scales must be 16-byte aligned");
  CUtensorMap ma, mb;
  if (int e = make_codes_map(&ma, a_codes, M, K, lda)) return e;
  if (int e = make_codes_map(&mb, b_codes, N, K, ldb)) return e;
  GemmArgs p{a_scales, b_scales, a_g, b_g, c, M, N, K, ldc, K / 64};
  if (int e = set_smem_attr((const void*)gemm_nvf4_kernel, gemm::SMEM_BYTES)) return e;
  dim3 grid((M + 127) / 128, (N + 127) / 128);
  gemm_nvf4_kernel<<<grid, gemm::THREADS, gemm::SMEM_BYTES, reinterpret_cast<cudaStream_t>(stream)>>>(ma, mb, p);
  return check_launch("gemm_nvf4_kernel");
}
