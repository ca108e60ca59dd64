// qkv_quant.cu -- a Q or K projection fused with RoPE and the NVFP4 row
// quantizer: packed attention operands straight from the hidden states.
//
// The reference's patched attention runs q_proj / k_proj (bf16 linear,
// llama_patch.py:147-149), quantizes the 2-D views [B*T, H*D] row-wise with a
// per-token global scale (llama_patch.py:167-194) and applies RoPE
// (llama_patch.py:210).  This path applies RoPE first and quantizes the
// rotated values (the FP4 tensor cores need FP4 operands after the rotation):
//
//   y   = bf16(x W^T)                                   (fp32 accumulate)
//   z   = bf16(bf16(y cos) + bf16(rotate_half(y) sin))  (HF apply_rotary_pos_emb
//                                                         in bf16, op for op)
//   codes, E4M3 scales, g = the row quantizer on z      (g = max_row |z|,
//                                                         fp4_quant_utils.py:118-169)
//
// written in the layout the attention kernel loads: codes [M][H*D/2], scales
// in tcgen05 atoms, g [M] (M = B*T tokens, T a multiple of 128).
//
// A tile is 128 tokens x hpc heads (hpc = 4, or H when H < 4; up to 512 fp32
// TMEM columns), computed with tcgen05 kind::f16 (bf16 operands staged by
// TMA, 64B swizzle, 4-stage ring).  The per-token global scale spans all H
// heads, i.e. the H/hpc tiles of a 128-token block: each tile stages its
// rotated bf16 values in shared memory, folds its row maxima into g with an
// atomic maximum, and quantizes its own columns once every tile of the block
// has added its maxima (a counter in global memory).  A persistent
// cooperative grid runs the tiles on every SM (thread-block clusters of H/4
// CTAs would leave SMs of each GPC idle: 15 clusters of 8 fit at once).  No
// bf16 Q/K tensor goes to HBM.  Every wait is bounded; a CTA whose wait gave
// up stops at the next tile barrier.
#include <cuda.h>
#include <cuda_bf16.h>

#include "common.cuh"
#include "fp4attn.h"
#include "sm100.cuh"
#include "status.h"
#include "tmap.h"

namespace fp4 {

FP4_DEFINE_STATUS_READER(qkv_status)

namespace {
namespace qkv {
constexpr int BM = 128, HD = 128, HPC = 4, BN = HPC * HD, BK = 32;  // BK: bf16 elements = 64 bytes per row
constexpr int STAGES = 4;
constexpr int X_BYTES = BM * BK * 2;             // 8 KB
constexpr int W_BYTES = BN * BK * 2;             // 32 KB
constexpr int STAGE_BYTES = X_BYTES + W_BYTES;   // 40 KB
constexpr int RING_BYTES = STAGES * STAGE_BYTES;  // 160 KB
constexpr int E_LD = BN * 2 + 16;  // staged row (bytes): 16 bytes of padding spread the rows over the banks
constexpr int E_BYTES = BM * E_LD;
static_assert(E_BYTES <= RING_BYTES, "the staged rows reuse the ring");
constexpr int AUX_BYTES = 2048;  // barriers, TMEM slot, row maxima, reciprocal table
constexpr int SMEM_BYTES = RING_BYTES + AUX_BYTES + 1024;
constexpr int THREADS = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue (one TMEM lane quarter each)
constexpr int MAX_TILES_PER_BLOCK = 16;  // head groups per token block (H <= 64)
constexpr uint32_t TMEM_COLS = 512;
}  // namespace qkv

struct QkvArgs {
  const __nv_bfloat16* cos;  // [M][HD]
  const __nv_bfloat16* sin;  // [M][HD]
  uint8_t* codes;            // [M][H*HD/2]
  uint8_t* scales;           // tcgen05 atoms, nkb4 groups per 128-row block
  float* g;                  // [M]
  int M, K, H;
  int nkb4;   // H*HD/64
  int hpc;    // heads per tile: 1, 2 or 4
  int csize;  // tiles per token block: H / hpc
};

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, f32 accumulate, M=128, K=16.
__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::f16 instruction descriptor with bf16 A/B (format 1 at [7,10) and [10,13)), f32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Global-memory flags of a token block (codes words, see the kernel's comment): acquire loads,
// release increments.
__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* w) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(w) : "memory");
  return v;
}
__device__ __forceinline__ void add_release_u32(unsigned int* w, unsigned int v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(w), "r"(v) : "memory");
}
// Bounded spin until *w >= target; false after the library's wait limit (records the site).
__device__ bool wait_count_u32(const unsigned int* w, unsigned int target, unsigned int site) {
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 0;; ++i) {
    if (ld_acquire_u32(w) >= target) return true;
    if ((i & 63) == 63) {
      if (dev_failed()) return false;
      if (globaltimer() - t0 > kWaitNs) {
        dev_fail(site);
        return false;
      }
    }
  }
}
// Order this thread's generic-proxy shared-memory accesses before later async-proxy (TMA) writes.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Wait for a bulk copy to land, whatever the failure flag says (bounded).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > kWaitNs) return;
}

// Persistent cooperative grid: CTA c takes tiles c, c + gridDim.x, ... of 128 tokens x hpc heads,
// the hpc-head groups of a token block consecutive, so a block's tiles run side by side.
// Per tile: main loop (TMA ring -> tcgen05), epilogue (RoPE into bf16 rows staged in the ring,
// the rows' maxima folded into g by an order-free atomic maximum), then the token block's
// hand-off: each tile increments the block's arrival word and waits until all csize tiles of the
// block have arrived, reads the finished g and quantizes its own columns; it then increments the
// departure word.  The two words are the first 8 code bytes of the block's first token (zeroed by
// the host); the block's head-group-0 tile, which owns those bytes, writes them last, once every
// tile of the block has departed.  Cooperative residency makes the waits safe: a tile waits only
// on tiles of its own block, whose CTAs each finish a strictly earlier tile first.
__global__ void __launch_bounds__(qkv::THREADS, 1)
    qkv_rope_quant_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                          QkvArgs p) {
  using namespace qkv;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + RING_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* s_ok = reinterpret_cast<volatile int*>(tmem_slot + 1);  // the token block's hand-off completed
  float* rcp_tab = reinterpret_cast<float*>(sm + RING_BYTES + 256);      // [128]
  const int warp = threadIdx.x / 32;
  const int ncols = p.hpc * HD;                   // output columns of a tile
  const int nrows_w = ncols < 256 ? ncols : 256;  // W rows per TMA box and per MMA (N)
  const int nw = ncols / nrows_w;                 // W boxes (and MMAs per K step)
  const uint32_t stage_tx = (uint32_t)(X_BYTES + ncols * BK * 2);
  const int ksteps = p.K / BK;
  const int tiles = (p.M / BM) * p.csize;
  const int64_t code_ld = (int64_t)p.H * HD / 2;  // code bytes per token

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1), mbar_init(&empty[s], 1);
    mbar_init(acc_full, 1);
    fence_barrier_init();
  }
  if (threadIdx.x < 128) {
    // correctly rounded 1/s for every non-negative E4M3 scale byte (0 -> 0, get_reciprocal)
    const float s = e4m3_to_f32((uint8_t)threadIdx.x);
    rcp_tab[threadIdx.x] = s == 0.0f ? 0.0f : __frcp_rn(s);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  int issued = 0;  // producer: k-steps issued in all (ring position across tiles)
  int fail = 0;    // this thread's wait gave up; the CTA stops at the next tile barrier (bar.red.or)

  for (int t = blockIdx.x, nt = 0; t < tiles; t += gridDim.x, ++nt) {
    const int tb = t / p.csize, hg = t % p.csize;
    const int m0 = tb * BM;
    const int n0 = hg * ncols;  // first output column: heads hpc*hg ..
    const int kg0 = nt * ksteps;  // this tile's first k-step in the ring's numbering
    unsigned int* flags = reinterpret_cast<unsigned int*>(p.codes + (int64_t)m0 * code_ld);  // [0] arrivals, [1] departures
    if (warp == 0) {
      // ----------------------------------------------- producer: X and W tiles
      if (elect_one_lane()) {
        if (nt == 0) {
          tma_prefetch_desc(&tmX);
          tma_prefetch_desc(&tmW);
        }
        for (int ks = 0; ks < ksteps; ++ks) {
          const int kg = kg0 + ks, s = kg % STAGES;
          if (kg >= STAGES && !mbar_wait(&empty[s], ((kg / STAGES) - 1) & 1, 0x601)) {
            fail = 1;
            break;
          }
          uint8_t* st = sm + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], stage_tx);
          tma_load_2d(st, &tmX, &full[s], ks * BK, m0);
          for (int i = 0; i < nw; ++i)
            tma_load_2d(st + X_BYTES + i * nrows_w * BK * 2, &tmW, &full[s], ks * BK, n0 + i * nrows_w);
          issued = kg + 1;
        }
      }
    } else if (warp == 1) {
      // ----------------------------------------------------------- MMA issue
      if (elect_one_lane()) {
        tc_fence_after();  // the previous tile's TMEM reads are done (CTA barrier below)
        const uint32_t idesc = idesc_bf16(BM, nrows_w);
        for (int ks = 0; ks < ksteps; ++ks) {
          const int kg = kg0 + ks, s = kg % STAGES;
          if (!mbar_wait(&full[s], (kg / STAGES) & 1, 0x602)) {
            fail = 1;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(sm + s * STAGE_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = smem_desc(st + kk * 32, 16, 512, kSwizzle64B);
            for (int i = 0; i < nw; ++i) {
              const uint64_t bd = smem_desc(st + X_BYTES + i * nrows_w * BK * 2 + kk * 32, 16, 512, kSwizzle64B);
              mma_bf16_ss(tmem + i * nrows_w, ad, bd, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
            }
          }
          tc_commit(&empty[s]);
        }
        tc_commit(acc_full);  // also on failure, so that the epilogue's wait ends once the MMAs are done
      }
    } else {
      // ------------------------------------------------ epilogue: RoPE, row max
      const int quarter = warp & 3;
      const int r = quarter * 32 + (threadIdx.x & 31);  // tile row == TMEM lane
      const int m = m0 + r;
      const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
      if (!mbar_wait(acc_full, nt & 1, 0x603)) fail = 1;
      tc_fence_after();
      if (!fail) {
        uint8_t* erow = sm + r * E_LD;
        const __nv_bfloat16* crow = p.cos + (int64_t)m * HD;
        const __nv_bfloat16* srow = p.sin + (int64_t)m * HD;
        float mx = 0.0f;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {  // dims 32c..32c+31 and their RoPE partners 64+32c..
          float c1[32], s1[32], c2[32], s2[32];
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            const uint4 a = *reinterpret_cast<const uint4*>(crow + 32 * c + i);
            const uint4 b = *reinterpret_cast<const uint4*>(srow + 32 * c + i);
            const uint4 a2 = *reinterpret_cast<const uint4*>(crow + 64 + 32 * c + i);
            const uint4 b2 = *reinterpret_cast<const uint4*>(srow + 64 + 32 * c + i);
            const __nv_bfloat16* ea = reinterpret_cast<const __nv_bfloat16*>(&a);
            const __nv_bfloat16* eb = reinterpret_cast<const __nv_bfloat16*>(&b);
            const __nv_bfloat16* ea2 = reinterpret_cast<const __nv_bfloat16*>(&a2);
            const __nv_bfloat16* eb2 = reinterpret_cast<const __nv_bfloat16*>(&b2);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              c1[i + k] = __bfloat162float(ea[k]);
              s1[i + k] = __bfloat162float(eb[k]);
              c2[i + k] = __bfloat162float(ea2[k]);
              s2[i + k] = __bfloat162float(eb2[k]);
            }
          }
#pragma unroll 1
          for (int j = 0; j < p.hpc; ++j) {
            uint32_t x1[32], x2[32];
            tmem_ld32(tmem + lane_base + j * HD + 32 * c, x1);
            tmem_ld32(tmem + lane_base + j * HD + 64 + 32 * c, x2);
            tmem_ld_wait();
            uint32_t o1[16], o2[16];  // bf16 pairs
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              float z1[2], z2[2];
#pragma unroll
              for (int k = 0; k < 2; ++k) {
                const float a1 = bf16r(__uint_as_float(x1[i + k]));  // y = bf16(x W^T)
                const float a2 = bf16r(__uint_as_float(x2[i + k]));
                // rotate_half(y) = [-y2, y1]; z = bf16(bf16(y cos) + bf16(rotate_half(y) sin))
                z1[k] = bf16r(__fadd_rn(bf16r(__fmul_rn(a1, c1[i + k])), bf16r(__fmul_rn(-a2, s1[i + k]))));
                z2[k] = bf16r(__fadd_rn(bf16r(__fmul_rn(a2, c2[i + k])), bf16r(__fmul_rn(a1, s2[i + k]))));
              }
              mx = nanmax(mx, nanmax(absmax3(z1[0], z1[1], z2[0]), fabsf(z2[1])));
              const __nv_bfloat162 h1 = __floats2bfloat162_rn(z1[0], z1[1]);
              const __nv_bfloat162 h2 = __floats2bfloat162_rn(z2[0], z2[1]);
              o1[i / 2] = *reinterpret_cast<const uint32_t*>(&h1);
              o2[i / 2] = *reinterpret_cast<const uint32_t*>(&h2);
            }
            uint4* e1 = reinterpret_cast<uint4*>(erow + (j * HD + 32 * c) * 2);
            uint4* e2 = reinterpret_cast<uint4*>(erow + (j * HD + 64 + 32 * c) * 2);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              e1[q] = make_uint4(o1[4 * q], o1[4 * q + 1], o1[4 * q + 2], o1[4 * q + 3]);
              e2[q] = make_uint4(o2[4 * q], o2[4 * q + 1], o2[4 * q + 2], o2[4 * q + 3]);
            }
          }
        }
        // per-token global scale over all H heads: g = max |z| (non-negative or NaN, NaN winning,
        // so the maximum of the bit patterns is the float maximum)
        atomicMax(reinterpret_cast<unsigned int*>(p.g) + m, __float_as_uint(mx));
        __threadfence();  // the maximum is in L2 before the block's arrival below
      }
      tc_fence_before();  // TMEM reads done before the next tile's MMAs
    }
    if (__syncthreads_or(fail)) break;  // main loop, staging and maxima of this tile done
    if (warp >= 2) {
      const int r = (warp & 3) * 32 + (threadIdx.x & 31);
      const int64_t m = m0 + r;
      if (threadIdx.x == 64) {
        add_release_u32(&flags[0], 1u);  // this tile's maxima are in g
        const bool ok = wait_count_u32(&flags[0], (unsigned)p.csize, 0x604);
        if (ok) add_release_u32(&flags[1], 1u);  // done with the arrival word
        *s_ok = ok ? 1 : 0;
        if (!ok) fail = 1;
      }
      named_bar(1, 128);
      if (*s_ok) {
        // ---- NVFP4 row quantizer on this tile's columns (fp4_quant_utils.py:118-169, fp32 arithmetic)
        const uint8_t* erow = sm + r * E_LD;
        // global_scale_aligned: g = rowmax, no division by global_sf_max; read at L2 (all tiles of the block added theirs)
        const float g = __ldcg(p.g + m);
        const float rg = g == 0.0f ? 0.0f : __frcp_rn(g);
        const float r6 = __frcp_rn(6.0f);
        uint4* crow = reinterpret_cast<uint4*>(p.codes + m * code_ld + n0 / 2);
        uint2 stash = make_uint2(0u, 0u);  // hg == 0, row 0: the flag words' bytes, written last
#pragma unroll 1
        for (int kb4 = 0; kb4 < ncols / 64; ++kb4) {  // 4 blocks of 16 = one scale word, 32 code bytes
          uint32_t words[8], sw = 0;
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const int kb = 4 * kb4 + b;
            const uint4 u0 = *reinterpret_cast<const uint4*>(erow + kb * 32);
            const uint4 u1 = *reinterpret_cast<const uint4*>(erow + kb * 32 + 16);
            const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
            float v[16];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              v[2 * k] = __fmul_rn(__uint_as_float(w[k] << 16), rg);
              v[2 * k + 1] = __fmul_rn(__uint_as_float(w[k] & 0xFFFF0000u), rg);
            }
            float am = 0.0f;
#pragma unroll
            for (int k = 0; k < 16; k += 4) am = nanmax(am, nanmax(absmax3(v[k], v[k + 1], v[k + 2]), fabsf(v[k + 3])));
            const uint8_t sb = e4m3_torch(__fmul_rn(am, r6));
            const float rs = rcp_tab[sb & 0x7F];
            const bool nan_block = (sb & 0x7F) == 0x7F;
#pragma unroll
            for (int k = 0; k < 16; k += 2) {
              // x * recip(s) + 0: one rounding; + 0 turns -0.0 into +0.0 (torch.sign(-0.0) == 0)
              const uint32_t byte = nan_block ? 0u : e2m1x2(__fmaf_rn(v[k], rs, 0.0f), __fmaf_rn(v[k + 1], rs, 0.0f));
              if (k % 8 == 0) words[2 * b + k / 8] = 0u;
              words[2 * b + k / 8] |= byte << (8 * ((k / 2) % 4));
            }
            sw |= (uint32_t)sb << (8 * b);
          }
          if (hg == 0 && r == 0 && kb4 == 0) {
            stash = make_uint2(words[0], words[1]);
            reinterpret_cast<uint2*>(crow)[1] = make_uint2(words[2], words[3]);
          } else {
            crow[2 * kb4] = make_uint4(words[0], words[1], words[2], words[3]);
          }
          crow[2 * kb4 + 1] = make_uint4(words[4], words[5], words[6], words[7]);
          const int kbg = n0 / 16 + 4 * kb4;  // first of the four global blocks (multiple of 4)
          *reinterpret_cast<uint32_t*>(p.scales + sf_tcgen05_offset(m, kbg, p.nkb4)) = sw;
        }
        if (hg == 0 && r == 0) {
          // every tile of the block has read the arrival word: its bytes can become codes
          if (wait_count_u32(&flags[1], (unsigned)p.csize, 0x605)) *reinterpret_cast<uint2*>(crow) = stash;
          else fail = 1;
        }
      }
      fence_proxy_async_smem();  // staged rows read before the next tile's TMA writes the ring
    }
    if (__syncthreads_or(fail)) break;  // the ring is free again
  }
  if (warp == 0 && elect_one_lane()) {
    // on a failure, nothing of the ring may still be in flight when the CTA exits
    for (int kg = issued > STAGES ? issued - STAGES : 0; kg < issued; ++kg)
      mbar_drain(&full[kg % STAGES], (kg / STAGES) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace
}  // namespace fp4

using namespace fp4;

extern "C" int fp4qkv_rope_quant(const void* x, const void* w, const void* cos, const void* sin, int M, int K, int H,
                                 int T, uint8_t* codes, uint8_t* scales, float* g, void* stream) {
  using namespace qkv;
  clear_error();
  if (!x || !w || !cos || !sin || !codes || !scales || !g) return set_error(FP4ATTN_ERR_ARG, "null pointer");
  if (M <= 0 || K <= 0 || H <= 0 || T <= 0) return set_error(FP4ATTN_ERR_ARG, "bad shape");
  if (T % BM || M % T) return set_error(FP4ATTN_ERR_UNSUPPORTED, "T must be a multiple of %d and divide M", BM);
  if (K % BK) return set_error(FP4ATTN_ERR_UNSUPPORTED, "the hidden size must be a multiple of %d", BK);
  const int hpc = H >= HPC ? HPC : H;
  if (H % hpc || hpc == 3 || H / hpc > MAX_TILES_PER_BLOCK)
    return set_error(FP4ATTN_ERR_UNSUPPORTED, "heads must be 1, 2 or a multiple of %d, at most %d", HPC,
                     HPC * MAX_TILES_PER_BLOCK);
  if (((uintptr_t)x | (uintptr_t)w | (uintptr_t)cos | (uintptr_t)sin | (uintptr_t)codes | (uintptr_t)scales |
       (uintptr_t)g) % 16)
    return set_error(FP4ATTN_ERR_ARG, "buffers must be 16-byte aligned");
  CUtensorMap mx, mw;
  if (int e = encode_tiled_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, BK,
                              BM, CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  const int nrows_w = hpc * HD < 256 ? hpc * HD : 256;
  if (int e = encode_tiled_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w, (uint64_t)K, (uint64_t)H * HD, (uint64_t)K * 2,
                              BK, nrows_w, CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  const int csize = H / hpc;
  QkvArgs a{reinterpret_cast<const __nv_bfloat16*>(cos), reinterpret_cast<const __nv_bfloat16*>(sin), codes, scales,
            g, M, K, H, H * HD / 64, hpc, csize};
  if (int e = set_smem_attr((const void*)qkv_rope_quant_kernel, SMEM_BYTES)) return e;
  int dev = 0, sms = 0, per_sm = 0, coop = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qkv_rope_quant_kernel, THREADS, SMEM_BYTES) !=
          cudaSuccess ||
      per_sm < 1 || !coop)
    return set_error(FP4ATTN_ERR_CUDA, "cooperative launch of qkv_rope_quant_kernel unavailable");
  const int tiles = (M / BM) * csize;
  const int grid = tiles < per_sm * sms ? tiles : per_sm * sms;
  if (grid < csize) return set_error(FP4ATTN_ERR_UNSUPPORTED, "fewer resident CTAs than tiles per token block");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // g accumulates the per-token maxima; the two flag words of each token block (the first 8 code
  // bytes of its first token) start at zero
  if (cudaMemsetAsync(g, 0, (size_t)M * sizeof(float), st) != cudaSuccess ||
      cudaMemset2DAsync(codes, (size_t)BM * H * HD / 2, 0, 8, (size_t)(M / BM), st) != cudaSuccess)
    return set_error(FP4ATTN_ERR_CUDA, "memset: %s", cudaGetErrorString(cudaGetLastError()));
  void* args[] = {&mx, &mw, &a};
  if (cudaLaunchCooperativeKernel((const void*)qkv_rope_quant_kernel, dim3((unsigned)grid), dim3(THREADS), args,
                                  SMEM_BYTES, st) != cudaSuccess)
    return check_launch("qkv_rope_quant_kernel");
  return check_launch("qkv_rope_quant_kernel");
}
