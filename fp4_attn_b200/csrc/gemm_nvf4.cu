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
// Two kernels.  gemm_nvf4_persistent (when B's 128-row blocks pair up): one
// CTA per SM walks 128x256 output tiles; warp 0 issues TMA (codes, 128B
// swizzle) and bulk copies (scale atoms) into a 4-stage ring that runs ahead
// across tiles, warp 1 copies the scale atoms into TMEM (tcgen05.cp) and
// issues tcgen05.mma kind::mxf4nvf4 M128 N256 (K = 64 per instruction, 4 per
// 256-wide stage) into a 256-column fp32 TMEM accumulator, and eight epilogue
// warps take the accumulator into registers, release it, then apply the
// global scales and store while the next tile accumulates.  gemm_nvf4_kernel
// (any N): one CTA per 128x128 tile, two CTAs per SM, the same roles with a
// 3-stage ring and four epilogue warps.
#include <cuda.h>

#include "common.cuh"
#include "sm100.cuh"
#include "status.h"
#include "tmap.h"

namespace fp4 {

namespace gemm {
constexpr int BM = 128, BK = 256;  // BK in elements (128 bytes of codes per row)
constexpr int THREADS = 192;
constexpr int SF_BYTES = 4 * 512;  // 4 atoms (one per K=64 chunk) of 128 rows x 4 scales
// gemm_nvf4_kernel's tiles: NB = 1 block of 128 rows of B per tile, two CTAs per SM (one's
// epilogue overlaps the other's main loop)
template <int NB>
struct Cfg {
  static constexpr int BN = 128 * NB;
  static constexpr int STAGES = 3;
  static constexpr int A_BYTES = BM * BK / 2, B_BYTES = BN * BK / 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + (1 + NB) * SF_BYTES;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
  // accumulator BN columns, then per stage 16 SFA + 16 * NB SFB columns
  static constexpr uint32_t SF_COLS = 16 * (1 + NB);
  static constexpr uint32_t TMEM_COLS = NB == 1 ? 256 : 512;
  static_assert(BN + STAGES * SF_COLS <= TMEM_COLS, "TMEM columns");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};
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

template <int NB>
__global__ void __launch_bounds__(gemm::THREADS, 2)
    gemm_nvf4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs p) {
  using namespace gemm;
  static_assert(NB == 1, "two CTAs per SM");
  using C = Cfg<NB>;
  constexpr int STAGES = C::STAGES, A_BYTES = C::A_BYTES, B_BYTES = C::B_BYTES, STAGE_BYTES = C::STAGE_BYTES;
  constexpr int BN = C::BN;
  constexpr uint32_t TMEM_COLS = C::TMEM_COLS;
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
  const uint32_t acc = tmem;  // columns [0, BN)

  if (warp == 0 && elect_one_lane()) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int k = 0; k < ksteps; ++k) {
      const int s = k % STAGES;
      if (k >= STAGES && !mbar_wait(&empty[s], ((k / STAGES) - 1) & 1, 0x101)) break;
      uint8_t* st = smem + s * STAGE_BYTES;
      mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
      tma_load_2d(st, &tmA, &full[s], k * (BK / 2), m0);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)  // 128 B rows, so the blocks continue one operand layout
        tma_load_2d(st + A_BYTES + nb * (B_BYTES / NB), &tmB, &full[s], k * (BK / 2), n0 + 128 * nb);
      bulk_load(st + A_BYTES + B_BYTES, p.sfa + ((int64_t)(m0 / 128) * p.nkb4 + k * 4) * 512, SF_BYTES, &full[s]);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
        bulk_load(st + A_BYTES + B_BYTES + (1 + nb) * SF_BYTES,
                  p.sfb + ((int64_t)(n0 / 128 + nb) * p.nkb4 + k * 4) * 512, SF_BYTES, &full[s]);
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
      // scale atoms in TMEM: A's chunk a at sfa_t + 4a; B's chunk a at sfb_t + 4 * NB * a, its
      // 128-row blocks in consecutive groups of 4 columns (TMEM column 4 * (row / 128) + row % 128 / 32)
      const uint32_t sfa_t = tmem + BN + s * C::SF_COLS, sfb_t = sfa_t + 16;
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        tmem_cp_sf_atom(sfa_t + 4 * a, smem_desc(smem_u32(st + A_BYTES + B_BYTES + a * 512), 16, 128, kSwizzleNone));
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
          tmem_cp_sf_atom(sfb_t + 4 * NB * a + 4 * nb,
                          smem_desc(smem_u32(st + A_BYTES + B_BYTES + (1 + nb) * SF_BYTES + a * 512), 16, 128,
                                    kSwizzleNone));
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t ad = smem_desc(smem_u32(st) + kk * 32, 16, 1024, kSwizzle128B);
        const uint64_t bd = smem_desc(smem_u32(st + A_BYTES) + kk * 32, 16, 1024, kSwizzle128B);
        mma_nvf4(acc, ad, bd, idesc, sfa_t + 4 * kk, sfb_t + 4 * NB * kk, (k > 0 || kk > 0) ? 1u : 0u);
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

// Persistent 128x256 tiles: one CTA per SM walks the tiles t = blockIdx.x, + gridDim.x, ... (M
// tile fastest, so consecutive tiles share the B block and the CTAs in flight share all of A in L2).
// Warp 0 runs the TMA ring ahead across tile boundaries, warp 2 copies each stage's twelve scale
// atoms into TMEM, warp 1 issues the MMAs, and eight epilogue warps (two per TMEM lane quarter,
// one per 128-column half) move the accumulator into registers, hand it back to the MMA warp at
// once (acc_empty) and scale and store while the next tile's main loop runs.  The atom copies
// have their own warp because the tensor pipe takes them in issue order from one thread (~50
// cycles each, twelve per stage against four ~134-cycle MMAs) but overlaps them with another
// thread's MMAs (measured: 64 copies from a second warp leave a stream of 64 MMAs unslowed); the
// copier commits sf_full[s] once a stage's atoms are in TMEM, which the MMA warp waits for.
namespace gemmp {
constexpr int NB = 2, BN = 256, STAGES = 4;
constexpr int THREADS = 96 + 256;
constexpr int EPI_WARPS = 8;  // warps 3..10
constexpr int A_BYTES = gemm::BM * gemm::BK / 2, B_BYTES = BN * gemm::BK / 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + (1 + NB) * gemm::SF_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr uint32_t SF_COLS = 16 * (1 + NB);
constexpr uint32_t TMEM_COLS = 512;
static_assert(BN + STAGES * SF_COLS <= TMEM_COLS, "TMEM columns");
static_assert(SMEM_BYTES <= 232448, "shared memory");
}  // namespace gemmp

__global__ void __launch_bounds__(gemmp::THREADS, 1)
    gemm_nvf4_persistent(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs p) {
  using namespace gemmp;
  constexpr int BM = gemm::BM, BK = gemm::BK, SF_BYTES = gemm::SF_BYTES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drained = acc_empty + 1;
  uint64_t* sf_full = drained + 1;        // [STAGES] the stage's scale atoms are in TMEM (copier's commit)
  uint64_t* cp_drained = sf_full + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(cp_drained + 1);
  // set when a wait gave up; every role then stops at its next tile boundary
  volatile uint32_t* failed = tmem_slot + 1;

  const int warp = threadIdx.x / 32;
  const int ksteps = p.K / BK;
  const int mt_count = (p.M + BM - 1) / BM;
  const int tiles = mt_count * ((p.N + BN - 1) / BN);

  if (threadIdx.x == 0) {
    *failed = 0u;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, EPI_WARPS);
    mbar_init(drained, 1);
    for (int s = 0; s < STAGES; ++s) mbar_init(&sf_full[s], 1);
    mbar_init(cp_drained, 1);
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
  const uint32_t acc = tmem;  // columns [0, 256)

  if (warp == 0 && elect_one_lane()) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    int it = 0;  // k-steps issued by this CTA, across tiles
    for (int t = blockIdx.x; t < tiles && !*failed; t += gridDim.x) {
      const int m0 = (t % mt_count) * BM, n0 = (t / mt_count) * BN;
      for (int k = 0; k < ksteps; ++k, ++it) {
        const int s = it % STAGES;
        if (it >= STAGES && !mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, 0x111)) {
          *failed = 1u;
          break;
        }
        uint8_t* st = smem + s * STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
        tma_load_2d(st, &tmA, &full[s], k * (BK / 2), m0);
        tma_load_2d(st + A_BYTES, &tmB, &full[s], k * (BK / 2), n0);
        tma_load_2d(st + A_BYTES + B_BYTES / 2, &tmB, &full[s], k * (BK / 2), n0 + 128);
        bulk_load(st + A_BYTES + B_BYTES, p.sfa + ((int64_t)(m0 / 128) * p.nkb4 + k * 4) * 512, SF_BYTES, &full[s]);
        bulk_load(st + A_BYTES + B_BYTES + SF_BYTES, p.sfb + ((int64_t)(n0 / 128) * p.nkb4 + k * 4) * 512, SF_BYTES,
                  &full[s]);
        bulk_load(st + A_BYTES + B_BYTES + 2 * SF_BYTES, p.sfb + ((int64_t)(n0 / 128 + 1) * p.nkb4 + k * 4) * 512,
                  SF_BYTES, &full[s]);
      }
    }
  } else if (warp == 1 && elect_one_lane()) {
    const uint32_t idesc = idesc_nvf4(BM, BN);
    int it = 0, nt = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++nt) {
      // the epilogue warps have moved the previous tile's accumulator out of TMEM
      if (nt > 0 && !mbar_wait(acc_empty, (nt - 1) & 1, 0x112)) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int k = 0; k < ksteps; ++k, ++it) {
        const int s = it % STAGES;
        // the copier waited for the stage's TMA before its atom copies: their commit covers both
        if (!mbar_wait(&sf_full[s], (it / STAGES) & 1, 0x113)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint8_t* st = smem + s * STAGE_BYTES;
        const uint32_t sfa_t = tmem + BN + s * SF_COLS, sfb_t = sfa_t + 16;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = smem_desc(smem_u32(st) + kk * 32, 16, 1024, kSwizzle128B);
          const uint64_t bd = smem_desc(smem_u32(st + A_BYTES) + kk * 32, 16, 1024, kSwizzle128B);
          mma_nvf4(acc, ad, bd, idesc, sfa_t + 4 * kk, sfb_t + 8 * kk, (k > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&empty[s]);
      }
      if (!ok) break;
      tc_commit(acc_full);
    }
    if (!ok) {
      *failed = 1u;
      __threadfence_block();
      tc_commit(acc_full);  // lets a waiting epilogue see the flag once the issued MMAs are done
    }
    // no MMA of this CTA is in flight when TMEM is released, on every path
    tc_commit(drained);
    mbar_wait(drained, 0, 0x115);
  } else if (warp == 2) {
    // ------------------------------------------------- scale atoms: shared memory -> TMEM
    if (elect_one_lane()) {
      int it = 0;
      for (int t = blockIdx.x; t < tiles && !*failed; t += gridDim.x) {
        for (int k = 0; k < ksteps; ++k, ++it) {
          const int s = it % STAGES;
          // the TMA for this use of the stage is issued only after the MMAs of its previous use
          // (empty[s]), so the stage's TMEM atom slot is free once the stage is full
          if (!mbar_wait(&full[s], (it / STAGES) & 1, 0x116)) {
            *failed = 1u;
            break;
          }
          tc_fence_after();
          const uint8_t* st = smem + s * STAGE_BYTES;
          const uint32_t sfa_t = tmem + BN + s * SF_COLS, sfb_t = sfa_t + 16;
#pragma unroll
          for (int a = 0; a < 4; ++a) {
            tmem_cp_sf_atom(sfa_t + 4 * a, smem_desc(smem_u32(st + A_BYTES + B_BYTES + a * 512), 16, 128, kSwizzleNone));
            tmem_cp_sf_atom(sfb_t + 8 * a,
                            smem_desc(smem_u32(st + A_BYTES + B_BYTES + SF_BYTES + a * 512), 16, 128, kSwizzleNone));
            tmem_cp_sf_atom(sfb_t + 8 * a + 4,
                            smem_desc(smem_u32(st + A_BYTES + B_BYTES + 2 * SF_BYTES + a * 512), 16, 128,
                                      kSwizzleNone));
          }
          tc_commit(&sf_full[s]);
        }
      }
      // no copy of this CTA is in flight when TMEM is released
      tc_commit(cp_drained);
      mbar_wait(cp_drained, 0, 0x117);
    }
  } else if (warp >= 3) {
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int half = (warp - 3) >> 2;
    const int row = quarter * 32 + (threadIdx.x & 31);
    const bool vec_out = p.ldc % 4 == 0 && (uintptr_t)p.c % 16 == 0 && (uintptr_t)p.gb % 16 == 0;
    int nt = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++nt) {
      const bool ok = mbar_wait(acc_full, nt & 1, 0x114) && *failed == 0u;
      tc_fence_after();
      if (!ok) break;
      uint32_t r[128];
#pragma unroll
      for (int c = 0; c < 128; c += 32) {
        uint32_t* rc = r + c;
        tmem_ld32(acc + ((uint32_t)(quarter * 32) << 16) + half * 128 + c, *reinterpret_cast<uint32_t(*)[32]>(rc));
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(acc_empty);
      const int m0 = (t % mt_count) * BM, nb = (t / mt_count) * BN + half * 128;
      const int m = m0 + row;
      if (m < p.M) {
        const float ga = p.ga ? p.ga[m] : 1.0f;
        float* dst = p.c + (int64_t)m * p.ldc + nb;
        if (vec_out && nb + 128 <= p.N) {
#pragma unroll
          for (int j = 0; j < 128; j += 4) {
            const float4 gb = p.gb ? *reinterpret_cast<const float4*>(p.gb + nb + j) : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
            float4 o;
            o.x = __uint_as_float(r[j]) * ga * gb.x;
            o.y = __uint_as_float(r[j + 1]) * ga * gb.y;
            o.z = __uint_as_float(r[j + 2]) * ga * gb.z;
            o.w = __uint_as_float(r[j + 3]) * ga * gb.w;
            *reinterpret_cast<float4*>(dst + j) = o;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 128; ++j) {
            const int n = nb + j;
            if (n < p.N) {
              const float gb = p.gb ? p.gb[n] : 1.0f;
              dst[j] = __uint_as_float(r[j]) * ga * gb;
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
  // persistent 128x256 tiles when the 128-row blocks of B pair up (a third less operand traffic
  // per flop; every scale atom a tile reads then exists), else 128x128 tiles, two CTAs per SM
  if (((N + 127) / 128) % 2 == 0) {
    if (int e = set_smem_attr((const void*)gemm_nvf4_persistent, gemmp::SMEM_BYTES)) return e;
    const int tiles = ((M + 127) / 128) * ((N + 255) / 256);
    int sms = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = tiles < sms ? tiles : (sms > 0 ? sms : 148);
    gemm_nvf4_persistent<<<grid, gemmp::THREADS, gemmp::SMEM_BYTES, reinterpret_cast<cudaStream_t>(stream)>>>(ma, mb, p);
  } else {
    using C = gemm::Cfg<1>;
    if (int e = set_smem_attr((const void*)gemm_nvf4_kernel<1>, C::SMEM_BYTES)) return e;
    dim3 grid((M + 127) / 128, (N + C::BN - 1) / C::BN);
    gemm_nvf4_kernel<1><<<grid, gemm::THREADS, C::SMEM_BYTES, reinterpret_cast<cudaStream_t>(stream)>>>(ma, mb, p);
  }
  return check_launch("gemm_nvf4_kernel");
}
