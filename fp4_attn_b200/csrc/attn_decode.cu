// attn_decode.cu -- FP4 attention for one new query token per sequence over an
// NVFP4 KV cache (decode).
//
// The reference's patched attention (llama_patch.py:167-215) quantizes each
// call's new Q/K/V, appends the dequantized K/V to the HF cache and runs the
// eager attention with P fake-quant (llama_patch.py:57-105) over every cached
// key.  Here the cache holds the packed NVFP4 data of those same values:
//   K: codes [B][Hkv][Tmax][D/2], E4M3 scales per 16 dims [B][Hkv][Tmax][D/16],
//      per-token global scale g_k [B][Tmax] (row mode on the [B*q, Hkv*D] view);
//   V, dim-major: codes [B][Hkv][D][Tmax/2] (byte j of a channel holds
//      tokens 2j and 2j+1, the first in the low nibble), one E4M3 scale byte
//      per element [B][Hkv][D][Tmax] (V's blocks of 16 run along the tokens of
//      the call that appended them, so a token's scale is per channel),
//      per-token g_v [B][Tmax]; optionally the same scales once per 16-token
//      group [B][Hkv][D][Tmax/16] for a prefix of len16 tokens whose groups
//      each came from one block (a call that started on a group boundary with
//      whole blocks per sequence).  Chunks of 256 keys inside that prefix read
//      the 2 KB of group scales instead of 32 KB of per-element scales.
// Tmax is a multiple of 256, so every chunk of 256 keys is whole in memory.
// The query comes in the same packed form (row mode on its [B, Hq*D] view):
// codes [B][Hq*D/2], E4M3 scales [B][Hq*D/16], g_q [B].
//
// Work item = (chunk of 256 keys, b, KV head).  Three kernels, HBM-bound:
//  * scores: persistent CTAs stream their items' K (TMA codes, scales) through
//    a ring; S^T = K-hat Q-hat^T on tcgen05 kind::mxf4nvf4 straight from the
//    cache's NVFP4 data (the query heads of the KV head are the MMA's N = 16
//    columns), S = acc * g_q * g_k * scaling written per key, and each row's
//    maximum folded into an order-free atomic maximum;
//  * pv: a ring of V (a TMA tile of 128 channels x 256 keys), S and g_v;
//    the exact row max, e = exp2(S log2 e - m log2 e), the NVFP4 fake-quant of e
//    per 16 keys (as the prefill kernel does), then O-partial^T =
//    (code*scale)_v^T (P-hat * g_v)^T on tcgen05 kind::f16 with V-hat in
//    TMEM (exact in fp16) and P-hat * g_v as fp16 hi + lo rows in shared
//    memory (V's per-token g_v is not exact in fp16), fp32 accumulate in TMEM;
//  * combine: O = sum O-partial / sum l over the chunks, in a fixed order.
#include <stdint.h>

#include <algorithm>

#include "attn_softmax.cuh"
#include "common.cuh"
#include "fp4attn.h"
#include "sm100.cuh"
#include "status.h"
#include "tmap.h"

namespace fp4 {

FP4_DEFINE_STATUS_READER(decode_status)

namespace {

constexpr int DK_KEYS = 256;  // keys per work item
constexpr int DK_MAXG = 16;   // query heads per KV head
constexpr int DK_D = 128;     // head dim

struct DecodeArgs {
  const uint8_t* q_codes;   // [B][Hq*D/2]
  const uint8_t* q_scales;  // [B][Hq*D/16]
  const float* q_g;         // [B]
  const uint8_t* k_codes;
  const uint8_t* k_scales;
  const float* k_g;
  const uint8_t* v_codes;
  const uint8_t* v_scales;
  const float* v_g;
  const uint8_t* v_scales16;  // [B][Hkv][Tmax/16][D], read for chunks split < nsplit16
  int B, Hq, Hkv, len, Tmax, nsplit, nsplit16;
  float scaling;
  float* S;            // [B*Hq][nsplit*DK_KEYS]
  float* opart;        // [B*Hq][nsplit][D]
  float* lpart;        // [B*Hq][nsplit][4]: l of a chunk in four parts
  unsigned int* mrow;  // [B*Hq] row maximum of S (float bits, atomic; 0xFFFFFFFF = none yet)
  float* out;          // [B][Hq][D]
};

// Position of a work item (chunk `split` of KV head hk of sequence b, bk = b * Hkv + hk), advanced
// item by item without the integer divisions of recomputing it.
struct ItemPos {
  int bk, split, b, hk;
  __device__ __forceinline__ ItemPos(int item, const DecodeArgs& p)
      : bk(item / p.nsplit), split(item % p.nsplit), b(bk / p.Hkv), hk(bk % p.Hkv) {}
  __device__ __forceinline__ void next(const DecodeArgs& p) {
    if (++split == p.nsplit) {
      split = 0, ++bk;
      if (++hk == p.Hkv) hk = 0, ++b;
    }
  }
};


__device__ __forceinline__ uint32_t cvt_e4m3x2_f16x2(uint32_t two_bytes) {
  uint32_t r;
  asm("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(r) : "r"(two_bytes));
  return r;
}
// Four E2M1 code pairs (the bytes of w, lowest first) as fp16 pairs.
__device__ __forceinline__ void cvt4_e2m1x2_f16x2(uint32_t w, uint32_t* o) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w));
}
__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// order-preserving float maximum on the bit pattern (exact, order-free)
__device__ __forceinline__ void atomic_max_f32(unsigned int* a, float v) {
  if (!(v < 0.0f)) atomicMax(reinterpret_cast<int*>(a), __float_as_int(v));
  else atomicMin(a, __float_as_uint(v));
}
// Named barrier 1 over NW warps that also ANDs a flag over their threads (every warp sees the same answer)
template <int NW>
__device__ __forceinline__ bool consumers_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)ok), "r"(NW * 32)
      : "memory");
  return r != 0;
}

// Wait for a bulk copy to land before the CTA exits, whatever the failure flag says (bounded).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > kWaitNs) return;
}

__device__ __forceinline__ void item_range(int n, int& i0, int& i1) {
  i0 = (int)((int64_t)blockIdx.x * n / gridDim.x);
  i1 = (int)((int64_t)(blockIdx.x + 1) * n / gridDim.x);
}

// The producer lane of a ring: item it of this CTA goes to stage it % NS once
// the consumers released that stage's previous item; load(item, stage, bar)
// issues the bulk copies.  Before returning it waits (bounded) for the copies
// of the last items it issued, so none is in flight when the CTA exits.
template <int NS, typename Load>
__device__ __forceinline__ void produce(uint64_t* full, uint64_t* empty, uint8_t* ring, uint32_t stage_bytes,
                                        int i0, int i1, unsigned int site, Load load) {
  int issued = 0;
  for (int it = 0; it < i1 - i0; ++it) {
    const int s = it % NS;
    if (it >= NS && !mbar_wait(&empty[s], ((it / NS) - 1) & 1, site)) break;
    load(i0 + it, ring + (size_t)s * stage_bytes, &full[s]);
    issued = it + 1;
  }
  for (int it = issued > NS ? issued - NS : 0; it < issued; ++it) mbar_drain(&full[it % NS], (it / NS) & 1);
}

// ---------------------------------------------------------------- scores
// S^T[key][head] = K-hat Q-hat^T on tcgen05 kind::mxf4nvf4 (E2M1 codes and
// E4M3 block scales straight from the cache, fp32 accumulate in TMEM), one
// 256-key item = two 128-key tiles per MMA pair:
//  * warp 0 streams an item's K codes (TMA, 64-byte swizzle: the rows are
//    the MMA's A operand as stored) and its E4M3 scales into a ring;
//  * warp 1 writes the KV head's query rows (B operand, N = 16: heads >= G
//    zero) and their scale atoms when the KV head changes, turns each item's
//    scales into the tcgen05 atom layout (row r at (r % 32) * 16 +
//    (r / 32) * 4), and one lane issues the copies and MMAs into one of four
//    accumulators;
//  * warps 2-5, a TMEM lane (key) per thread: S = acc * g_q * g_k * scaling
//    (keys past len -inf), written with 32 consecutive keys per warp store,
//    and each head's running maximum, folded into the order-free atomic row
//    maximum when the KV head changes.
namespace dsc {
constexpr int NS = 4, NACC = 4;
constexpr int THREADS = 6 * 32;
constexpr uint32_t KC = DK_KEYS * DK_D / 2;   // codes: 256 rows x 64 B
constexpr uint32_t KS = DK_KEYS * DK_D / 16;  // scales: 256 rows x 8 B
constexpr uint32_t STAGE = KC + KS;
constexpr uint32_t OFF_ATOM = NS * STAGE;           // [NACC][tile][kk] atoms of 512 B
constexpr uint32_t OFF_Q = OFF_ATOM + NACC * 2048;  // 16 query rows x 64 B, 64-byte swizzle
constexpr uint32_t OFF_QSF = OFF_Q + 1024;          // [kk] query scale atoms
constexpr uint32_t SMEM = OFF_QSF + 1024 + 1024;    // + alignment slack
constexpr uint32_t T_SFA = 32 * NACC, T_SFB = T_SFA + 16 * NACC, TMEM_COLS = 256;
static_assert(STAGE % 1024 == 0 && T_SFB + 8 <= TMEM_COLS, "layout");
}  // namespace dsc

template <int MG>
__global__ void __launch_bounds__(dsc::THREADS) decode_scores_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                     DecodeArgs p) {
  using namespace dsc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[NS], empty[NS], acc_full[NACC], acc_free[NACC], qdrain, drained;
  __shared__ uint32_t tslot;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int G = p.Hq / p.Hkv;
  int i0, i1;
  item_range(p.nsplit * p.B * p.Hkv, i0, i1);
  const int n_items = i1 - i0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(&full[s], 1), mbar_init(&empty[s], 1);
    for (int i = 0; i < NACC; ++i) mbar_init(&acc_full[i], 1), mbar_init(&acc_free[i], 4);
    mbar_init(&qdrain, 1), mbar_init(&drained, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tslot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      produce<NS>(full, empty, sm, STAGE, i0, i1, 0x401, [&](int item, uint8_t* st, uint64_t* bar) {
        const int bk = item / p.nsplit, split = item % p.nsplit;
        const int64_t row = (int64_t)bk * p.Tmax + (int64_t)split * DK_KEYS;
        mbar_arrive_expect_tx(bar, STAGE);
        tma_load_2d(st, &tmK, bar, 0, (int)row);
        bulk_load(st + KC, p.k_scales + row * (DK_D / 16), KS, bar);
      });
    }
  } else if (warp == 1) {
    const uint32_t idesc = idesc_nvf4(128, 16);
    uint8_t* qs = sm + OFF_Q;
    uint8_t* qsf = sm + OFF_QSF;
    int cur = -1, nq = 0;
    bool ok = true;
    ItemPos pos(i0, p);
    for (int it = 0; it < n_items && ok; ++it, pos.next(p)) {
      const int bk = pos.bk;
      const int s = it % NS, ai = it % NACC;
      if (bk != cur) {
        // a new KV head: every MMA issued so far reads the old query rows; let them finish first
        if (cur >= 0) {
          if (lane == 0) tc_commit(&qdrain);
          ok = __all_sync(0xffffffffu, mbar_wait(&qdrain, nq & 1, 0x402));
          ++nq;
          if (!ok) break;
        }
        cur = bk;
        const int b = pos.b, hk = pos.hk;
        // query rows n < G (heads hk G + n), zero above; chunk c of row n at n * 64 + (c ^ (n / 2 % 4)) * 16
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int n = (lane + 32 * i) >> 2, c = lane & 3;
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (n < G)
            v = __ldg(reinterpret_cast<const uint4*>(p.q_codes + ((int64_t)b * p.Hq + hk * G + n) * (DK_D / 2)) + c);
          *reinterpret_cast<uint4*>(qs + n * 64 + ((c ^ ((n >> 1) & 3)) << 4)) = v;
        }
        // scale atoms of the query rows: row n, blocks 4 kk .. 4 kk + 3 at n * 16 in atom kk
#pragma unroll
        for (int i = 0; i < 2; ++i) reinterpret_cast<uint4*>(qsf)[lane + 32 * i] = make_uint4(0u, 0u, 0u, 0u);
        __syncwarp();
        if (lane < G) {
          const uint2 sc = __ldg(reinterpret_cast<const uint2*>(p.q_scales + ((int64_t)b * p.Hq + hk * G + lane) * (DK_D / 16)));
          reinterpret_cast<uint32_t*>(qsf)[lane * 4] = sc.x;
          reinterpret_cast<uint32_t*>(qsf + 512)[lane * 4] = sc.y;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          tc_fence_after();
          tmem_cp_sf_atom(tmem + T_SFB, smem_desc(smem_u32(qsf), 16, 128, kSwizzleNone));
          tmem_cp_sf_atom(tmem + T_SFB + 4, smem_desc(smem_u32(qsf + 512), 16, 128, kSwizzleNone));
        }
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (it / NS) & 1, 0x403));
      if (ok && it >= NACC) ok = __all_sync(0xffffffffu, mbar_wait(&acc_free[ai], ((it - NACC) / NACC) & 1, 0x404));
      if (!ok) break;
      // the item's K scales into atoms: key r + 128 t, blocks 4 kk .. 4 kk + 3
      const uint8_t* st = sm + (size_t)s * STAGE;
      uint8_t* at = sm + OFF_ATOM + ai * 2048;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int key = lane + 32 * j, t = key >> 7, r = key & 127;
        const uint2 sc = *reinterpret_cast<const uint2*>(st + KC + key * 8);
        const uint32_t off = (r & 31) * 16 + ((r >> 5) & 3) * 4;
        *reinterpret_cast<uint32_t*>(at + t * 1024 + off) = sc.x;
        *reinterpret_cast<uint32_t*>(at + t * 1024 + 512 + off) = sc.y;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        tc_fence_after();
        const uint32_t sfa = tmem + T_SFA + 16 * ai;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          tmem_cp_sf_atom(sfa + 4 * c, smem_desc(smem_u32(at + 512 * c), 16, 128, kSwizzleNone));
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int kk = 0; kk < 2; ++kk)
            mma_nvf4(tmem + 32 * ai + 16 * t, smem_desc(smem_u32(st + t * 8192) + kk * 32, 16, 512, kSwizzle64B),
                     smem_desc(smem_u32(qs) + kk * 32, 16, 512, kSwizzle64B), idesc, sfa + 8 * t + 4 * kk,
                     tmem + T_SFB + 4 * kk, kk > 0 ? 1u : 0u);
        tc_commit(&empty[s]);
        tc_commit(&acc_full[ai]);
      }
      __syncwarp();
    }
    if (lane == 0) {
      tc_commit(&drained);  // every copy and MMA issued completes before TMEM is released
      mbar_drain(&drained, 0);
    }
  } else {
    // ------------------------------------------------------------ S, row maxima
    const int quarter = warp & 3;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const int64_t ks = (int64_t)p.nsplit * DK_KEYS;
    int cur = -1;
    int64_t bh0 = 0;
    float gq = 0.0f;
    float mx[MG];
#pragma unroll
    for (int h = 0; h < MG; ++h) mx[h] = -INFINITY;
    auto flush = [&]() {
#pragma unroll
      for (int h = 0; h < MG; ++h) {
        if (h >= G) break;
        float v = mx[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) atomic_max_f32(&p.mrow[bh0 + h], v);
        mx[h] = -INFINITY;
      }
    };
    ItemPos pos(i0, p);
    for (int it = 0; it < n_items; ++it, pos.next(p)) {
      const int bk = pos.bk, split = pos.split, b = pos.b, hk = pos.hk, ai = it % NACC;
      if (bk != cur) {
        if (cur >= 0) flush();
        cur = bk;
        bh0 = (int64_t)b * p.Hq + hk * G;
        gq = p.q_g[b];
      }
      const int k0 = split * DK_KEYS + quarter * 32 + lane;  // this lane's key of tile 0 (+128: tile 1)
      const float gk0 = __ldg(p.k_g + (int64_t)b * p.Tmax + k0), gk1 = __ldg(p.k_g + (int64_t)b * p.Tmax + k0 + 128);
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[ai], (it / NACC) & 1, 0x405));
      tc_fence_after();
      if (!ok) break;
      uint32_t r0[16], r1[16];
      tmem_ld16(tmem + lane_base + 32 * ai, r0);
      tmem_ld16(tmem + lane_base + 32 * ai + 16, r1);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_free[ai]);
#pragma unroll
      for (int h = 0; h < MG; ++h) {
        if (h >= G) break;
        float* srow = p.S + (bh0 + h) * ks;
        const float s0 = k0 < p.len ? __fmul_rn(__fmul_rn(__fmul_rn(__uint_as_float(r0[h]), gq), gk0), p.scaling)
                                    : -INFINITY;
        const float s1 = k0 + 128 < p.len
                             ? __fmul_rn(__fmul_rn(__fmul_rn(__uint_as_float(r1[h]), gq), gk1), p.scaling)
                             : -INFINITY;
        srow[k0] = s0;
        srow[k0 + 128] = s1;
        mx[h] = fmaxf(mx[h], fmaxf(s0, s1));
      }
    }
    if (cur >= 0) flush();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// -------------------------------------------------------------------- pv
// O-partial^T[channel][head] = V-hat^T[channel][key] (P-hat g_v)^T[key][head]
// on tcgen05 (kind::f16, A from TMEM, fp32 accumulate in TMEM), one 256-key
// item at a time:
//  * V is dim-major in the cache, so an item's codes are one 128 x 128-byte
//    tile (a row per channel, TMA with the 128-byte swizzle) and TMEM lane d
//    (channel d) takes its own run of tokens: code byte j converts to the
//    fp16 pair (token 2j, token 2j+1) of A column j, times the pair's E4M3
//    scales (one group scale per 16 tokens inside the group prefix, per
//    element past it).  V-hat = code * scale is exact in fp16 (at most five
//    significant bits in [2^-10, 2688]).  Eight converter warps: TMEM lane
//    quarter = warp % 4, half of the item's tokens = the warpgroup.
//  * B = P-hat * g_v * 2^E as fp16 hi (rows [0, MG)) + lo (rows [MG, 2 MG)),
//    K-major with the 128-byte swizzle: g_v varies along the keys, so it
//    cannot be factored out, and hi + lo keep 22 significant bits; 2^E, one
//    power of two per item, puts the largest value just below 2^15 and is
//    taken back out of the partial exactly.  Eight P warps: a thread takes a
//    key pair and every other query head; e = exp2(S log2 e - m log2 e) and
//    the NVFP4 fake-quant of e per 16 keys (block maximum over eight lanes),
//    with the prefill kernel's arithmetic (packed fp32 pairs, ex2, the block
//    scale's reciprocal by rcp).  Each P warp writes its own quarter of l
//    (64 keys); no warp waits for another's bookkeeping.
//  * one thread issues an item's 16 MMAs (M = 128 channels, N = 2 MG rounded
//    up to 16, K = 16 keys) into one of two accumulators; the first four
//    converter warps write an item's partial, (hi + lo) 2^-E, after handing
//    over the next item's V-hat.
namespace dpv {
constexpr int NS = 4;               // ring stages
constexpr int CW0 = 2, NCW = 8;     // converter warps 2 .. 9 (2 .. 5 also write the partials)
constexpr int PW0 = 10, NPW = 8;    // P warps 10 .. 17
constexpr int THREADS = (PW0 + NPW) * 32;
constexpr uint32_t VC = DK_KEYS * DK_D / 2;       // codes [128 channels][128 B]
constexpr uint32_t VS16 = DK_D * (DK_KEYS / 16);  // group scales [128 channels][16]
constexpr uint32_t VG = DK_KEYS * 4;
constexpr uint32_t S1 = DK_KEYS * 4;              // S of one head
constexpr uint32_t T_A = 0, T_ACC = 256;          // TMEM: A buffers 0 / 128, accumulators 256 / 288
template <int MG>
struct Cfg {
  static constexpr int NP = 2 * MG < 16 ? 16 : 2 * MG;  // B rows (MMA N)
  static constexpr uint32_t STAGE = VC + VS16 + VG + MG * S1;
  static constexpr uint32_t KBLK = NP * 128;  // B rows of one 64-key block
  static constexpr uint32_t PB = 4 * KBLK;    // B of one item
  static constexpr uint32_t OFF_PB = NS * STAGE;
  static constexpr uint32_t SMEM = OFF_PB + 2 * PB + 1024;  // + alignment slack
  static_assert(STAGE % 1024 == 0, "every stage keeps the 1024-byte alignment of the swizzled tile");
  static_assert(NP <= 32, "two accumulators of NP columns at T_ACC");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};
}  // namespace dpv

template <int MG>
__global__ void __launch_bounds__(dpv::THREADS, 1)
    decode_pv_kernel(const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmVs,
                     DecodeArgs p) {
  using namespace dpv;
  using C = Cfg<MG>;
  constexpr int NH = MG / 2;  // query heads per P thread: hs, hs + 2, ...
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[NS], empty[NS], a_full[2], a_free[2], b_full[2], b_free[2], acc_full[2],
      acc_free[2], drained;
  __shared__ uint32_t tslot;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int G = p.Hq / p.Hkv;
  int i0, i1;
  item_range(p.nsplit * p.B * p.Hkv, i0, i1);
  const int n_items = i1 - i0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(&full[s], 1), mbar_init(&empty[s], NCW + NPW);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&a_full[i], NCW), mbar_init(&a_free[i], 1);
      mbar_init(&b_full[i], NPW), mbar_init(&b_free[i], 1);
      mbar_init(&acc_full[i], 1), mbar_init(&acc_free[i], 4);
    }
    mbar_init(&drained, 1);
    fence_barrier_init();
  }
  // B rows of heads >= G and rows >= 2 MG stay zero
  for (uint32_t i = threadIdx.x; i < 2 * C::PB / 16; i += THREADS)
    reinterpret_cast<uint4*>(sm + C::OFF_PB)[i] = make_uint4(0u, 0u, 0u, 0u);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 1) {
    tmem_alloc(&tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  // 2^E of an item: the largest g_v of its live keys, read by every warp that needs it (no cross-warp
  // exchange); P-hat * g_v * 2^E < 2^15 (P-hat <= 1.03125 < 2, g_v < 2^(e+1))
  auto item_exp = [&](const uint8_t* st, int nlive, float& up, float& down) {
    const float4* gv = reinterpret_cast<const float4*>(st + VC + VS16) + 2 * lane;  // keys 8 lane .. 8 lane + 7
    const float4 a = gv[0], b = gv[1];
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float g = 0.0f;  // g_v >= 0
    if (nlive >= DK_KEYS) {
      g = fmaxf(max3f(v[0], v[1], v[2]), max3f(v[3], v[4], max3f(v[5], v[6], v[7])));
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) g = 8 * lane + i < nlive ? fmaxf(g, v[i]) : g;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) g = fmaxf(g, __shfl_xor_sync(0xffffffffu, g, o));
    int E = 0;
    if (g > 0.0f) E = max(-100, min(100, 13 - (((__float_as_int(g) >> 23) & 0xFF) - 127)));
    up = __int_as_float((E + 127) << 23), down = __int_as_float((127 - E) << 23);
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmVs);
      produce<NS>(full, empty, sm, C::STAGE, i0, i1, 0x411, [&](int item, uint8_t* st, uint64_t* bar) {
        const int bk = item / p.nsplit, split = item % p.nsplit, b = bk / p.Hkv, hk = bk % p.Hkv;
        const int64_t ks = (int64_t)p.nsplit * DK_KEYS;
        const bool compact = split < p.nsplit16;
        mbar_arrive_expect_tx(bar, VC + (compact ? VS16 : 0u) + VG + (uint32_t)G * S1);
        tma_load_2d(st, &tmV, bar, split * (DK_KEYS / 2), bk * DK_D);
        if (compact) tma_load_2d(st + VC, &tmVs, bar, split * (DK_KEYS / 16), bk * DK_D);
        bulk_load(st + VC + VS16, p.v_g + (int64_t)b * p.Tmax + (int64_t)split * DK_KEYS, VG, bar);
        for (int g = 0; g < G; ++g)
          bulk_load(st + VC + VS16 + VG + g * S1,
                    p.S + ((int64_t)b * p.Hq + hk * G + g) * ks + (int64_t)split * DK_KEYS, S1, bar);
      });
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issue
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, C::NP);
      for (int it = 0; it < n_items; ++it) {
        const int a = it & 1;
        if (!mbar_wait(&a_full[a], (it >> 1) & 1, 0x412)) break;
        if (!mbar_wait(&b_full[a], (it >> 1) & 1, 0x413)) break;
        if (it >= 2 && !mbar_wait(&acc_free[a], ((it - 2) >> 1) & 1, 0x414)) break;
        tc_fence_after();
        const uint32_t pb = smem_u32(sm + C::OFF_PB + a * C::PB);
#pragma unroll
        for (int ks = 0; ks < DK_KEYS / 16; ++ks)
          mma_f16_ts(tmem + T_ACC + 32 * a, tmem + T_A + 128 * a + 8 * ks,
                     smem_desc(pb + (ks >> 2) * C::KBLK + (ks & 3) * 32, 16, 1024, kSwizzle128B), idesc,
                     ks > 0 ? 1u : 0u);
        tc_commit(&a_free[a]);
        tc_commit(&b_free[a]);
        tc_commit(&acc_full[a]);
      }
      tc_commit(&drained);  // every MMA issued completes before TMEM is released
      mbar_drain(&drained, 0);
    }
  } else if (warp < PW0) {
    // ------------------------------------------------ V-hat into TMEM; partials (warps 2-5)
    const int quarter = warp & 3, half = (warp - CW0) >> 2;
    const bool epi = half == 0;
    const int d = quarter * 32 + lane;  // channel == TMEM lane
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    float prev_down = 1.0f;
    // the partial of item i: (hi + lo) 2^-E of this lane's channel, while item i + 1's MMAs wait for their
    // operands
    auto epilogue = [&](int i, const ItemPos& q) {
      const int a = i & 1, split = q.split;
      const int64_t bh0 = (int64_t)q.b * p.Hq + q.hk * G;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[a], (i >> 1) & 1, 0x417));
      tc_fence_after();
      if (ok) {
        uint32_t r[32];
        if constexpr (C::NP == 16) {
          uint32_t r16[16];
          tmem_ld16(tmem + lane_base + T_ACC + 32 * a, r16);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 16; ++c) r[c] = r16[c];
        } else {
          tmem_ld32(tmem + lane_base + T_ACC + 32 * a, r);
          tmem_ld_wait();
        }
#pragma unroll
        for (int h = 0; h < MG; ++h)
          if (h < G)
            p.opart[((bh0 + h) * p.nsplit + split) * DK_D + d] =
                (__uint_as_float(r[h]) + __uint_as_float(r[MG + h])) * prev_down;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_free[a]);
    };
    ItemPos pos(i0, p), prev = pos;
    int it = 0;
    for (; it < n_items; ++it, prev = pos, pos.next(p)) {
      const int bk = pos.bk, split = pos.split;
      const int s = it % NS, a = it & 1;
      if (!mbar_wait(&full[s], (it / NS) & 1, 0x415)) break;
      if (it >= 2 && !mbar_wait(&a_free[a], ((it - 2) >> 1) & 1, 0x416)) break;
      tc_fence_after();
      const uint8_t* st = sm + (size_t)s * C::STAGE;
      const int nlive = min(DK_KEYS, p.len - split * DK_KEYS);
      float up, down;
      if (epi) item_exp(st, nlive, up, down);
      uint4 cw[4];  // this half's 64 code bytes: logical 16-byte chunks 4 half .. 4 half + 3 of the row
#pragma unroll
      for (int c = 0; c < 4; ++c)
        cw[c] = *reinterpret_cast<const uint4*>(st + d * 128 + (((4 * half + c) ^ (d & 7)) << 4));
      const uint32_t acol = tmem + lane_base + T_A + 128 * a + 64 * half;
      if (split < p.nsplit16) {
        // every key of the chunk is live; groups 8 half .. 8 half + 7 of the channel
        const uint2 g8 = *reinterpret_cast<const uint2*>(st + VC + d * 16 + 8 * half);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t gw = c < 2 ? g8.x : g8.y;
          const uint32_t b0 = (gw >> (16 * (c & 1))) & 0xFFu, b1 = (gw >> (16 * (c & 1) + 8)) & 0xFFu;
          const uint32_t s0 = cvt_e4m3x2_f16x2(b0 * 0x101u), s1 = cvt_e4m3x2_f16x2(b1 * 0x101u);
          const uint32_t w[4] = {cw[c].x, cw[c].y, cw[c].z, cw[c].w};
          uint32_t o[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) cvt4_e2m1x2_f16x2(w[q], o + 4 * q);
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = hmul2u(o[j], j < 8 ? s0 : s1);
          tmem_st16(acol + 16 * c, o);
        }
      } else {
        // per-element scales from the cache (L2); keys past len read scale 0, so V-hat is 0 there
        const uint8_t* vs = p.v_scales + ((int64_t)bk * DK_D + d) * p.Tmax + (int64_t)split * DK_KEYS + 128 * half;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint4 sc[2];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int n = nlive - (128 * half + 32 * c + 16 * i);  // live keys of these 16
            sc[i] = n > 0 ? __ldg(reinterpret_cast<const uint4*>(vs + 32 * c + 16 * i)) : make_uint4(0u, 0u, 0u, 0u);
            if (n < 16) {
              uint32_t* e = reinterpret_cast<uint32_t*>(&sc[i]);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int m = n - 4 * q;  // live bytes of word q
                e[q] = m >= 4 ? e[q] : m <= 0 ? 0u : e[q] & (0xFFFFFFFFu >> (32 - 8 * m));
              }
            }
          }
          const uint32_t w[4] = {cw[c].x, cw[c].y, cw[c].z, cw[c].w};
          const uint32_t sw[8] = {sc[0].x, sc[0].y, sc[0].z, sc[0].w, sc[1].x, sc[1].y, sc[1].z, sc[1].w};
          uint32_t o[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) cvt4_e2m1x2_f16x2(w[q], o + 4 * q);
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = hmul2u(o[j], cvt_e4m3x2_f16x2((sw[j >> 1] >> (16 * (j & 1))) & 0xFFFFu));
          tmem_st16(acol + 16 * c, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[a]);
      if (epi) {
        if (it >= 1) epilogue(it - 1, prev);
        prev_down = down;
      }
    }
    if (epi && it >= 1) epilogue(it - 1, prev);
  } else {
    // ---------------------------------------------------------------- P-hat and l
    const int pt = threadIdx.x - PW0 * 32;
    const int hs = pt >> 7, pair = pt & 127, k0 = 2 * pair;
    const float log2e = 1.4426950408889634f, r6 = __frcp_rn(6.0f);
    const uint64_t l2e2 = pk2(log2e, log2e);
    // B word of keys (k0, k0 + 1): 64-key block, byte (k0 & 63) * 2 of the 128-byte row, chunk swizzled by row & 7
    const uint32_t kb_off = (uint32_t)(k0 >> 6) * C::KBLK, wb = (uint32_t)(k0 & 63) * 2;
    auto bword = [&](int row) { return kb_off + row * 128 + ((((wb >> 4) ^ (row & 7)) << 4) | (wb & 15)); };
    uint64_t nml2[NH];  // -m log2 e of the thread's heads, as pairs
#pragma unroll
    for (int j = 0; j < NH; ++j) nml2[j] = pk2(0.0f, 0.0f);
    int cur = -1;
    ItemPos pos(i0, p);
    for (int it = 0; it < n_items; ++it, pos.next(p)) {
      const int bk = pos.bk, split = pos.split, b = pos.b, hk = pos.hk;
      const int64_t bh0 = (int64_t)b * p.Hq + hk * G;
      if (bk != cur) {
        cur = bk;
#pragma unroll
        for (int j = 0; j < NH; ++j)
          if (hs + 2 * j < G) {
            const float nm = -__fmul_rn(__uint_as_float(p.mrow[bh0 + hs + 2 * j]), log2e);
            nml2[j] = pk2(nm, nm);
          }
      }
      const int s = it % NS, par = it & 1;
      if (!mbar_wait(&full[s], (it / NS) & 1, 0x418)) break;
      const uint8_t* st = sm + (size_t)s * C::STAGE;
      const int nlive = min(DK_KEYS, p.len - split * DK_KEYS);
      const bool live0 = k0 < nlive, live1 = k0 + 1 < nlive;
      float up, down;
      item_exp(st, nlive, up, down);
      const float2 gv2 = *reinterpret_cast<const float2*>(st + VC + VS16 + 8 * pair);
      // g_v 2^E of the two keys (exact: 2^E is a power of two); 0 past len
      const uint64_t gu2 = pk2(live0 ? __fmul_rn(gv2.x, up) : 0.0f, live1 ? __fmul_rn(gv2.y, up) : 0.0f);
      const float* Ss = reinterpret_cast<const float*>(st + VC + VS16 + VG);
      uint64_t ee[NH];  // (e of key k0, e of key k0 + 1) per head
#pragma unroll
      for (int j = 0; j < NH; ++j) {
        const int h = hs + 2 * j;
        ee[j] = pk2(0.0f, 0.0f);
        if (h < G) {  // uniform over the warp
          // e = exp2(S log2 e - m log2 e), as the prefill kernel computes it
          const float2 s2 = *reinterpret_cast<const float2*>(Ss + h * DK_KEYS + k0);
          float t0, t1;
          upk2(fma2(pk2(s2.x, s2.y), l2e2, nml2[j]), t0, t1);
          const float e0 = live0 ? ex2(t0) : 0.0f, e1 = live1 ? ex2(t1) : 0.0f;
          ee[j] = pk2(e0, e1);
          // this warp's share of l (its 64 keys), one of four per head and chunk
          float l = e0 + e1;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
          if (lane == 0) p.lpart[((bh0 + h) * p.nsplit + split) * 4 + (pair >> 5)] = l;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);  // S and g_v are in registers
      // the B buffer is free once the MMAs of item it - 2 have read it
      if (it >= 2 && !mbar_wait(&b_free[par], ((it - 2) >> 1) & 1, 0x419)) break;
      uint8_t* pb = sm + C::OFF_PB + par * C::PB;
#pragma unroll
      for (int j = 0; j < NH; ++j) {
        const int h = hs + 2 * j;
        if (h >= G) continue;  // uniform over the warp
        float e0, e1;
        upk2(ee[j], e0, e1);
        float am = fmaxf(e0, e1);  // block of 16 keys = 8 consecutive lanes
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        // the block's E4M3 scale (fp16 pair, exact) and its reciprocal by rcp, as the prefill kernel
        const uint32_t s2 = e4m3_f16x2(e4m3_satfinite(__fmul_rn(am, r6)) & 127);
        const float sv = __half2float(__ushort_as_half((unsigned short)(s2 & 0xFFFFu)));
        float rs;
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(rs) : "f"(sv));
        rs = sv == 0.0f ? 0.0f : rs;
        float x0, x1;
        upk2(mul2(ee[j], pk2(rs, rs)), x0, x1);
        const float2 ph = f16x2_to_f32(quant_pair_cvt(x0, x1, s2));  // P-hat = code * scale, exact
        upk2(mul2(pk2(ph.x, ph.y), gu2), x0, x1);
        const __half2 hi = __floats2half2_rn(x0, x1);
        const float2 hf = __half22float2(hi);
        *reinterpret_cast<__half2*>(pb + bword(h)) = hi;
        *reinterpret_cast<__half2*>(pb + bword(MG + h)) = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&b_full[par]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// O = sum over chunks of O-partial / sum of l.  One CTA per (b, query head):
// group r of 32 threads sums chunks r, r + 16, r + 32, ... (4 dims per thread,
// 16-byte loads, every load of the group issued before the adds), then the
// sixteen group sums are added in a fixed order.
constexpr int CB_GROUPS = 16;
__global__ void __launch_bounds__(CB_GROUPS * 32) decode_combine_kernel(DecodeArgs p) {
  __shared__ float4 osum[CB_GROUPS][DK_D / 4];
  __shared__ float lsum[CB_GROUPS];
  const int bh = blockIdx.x, r = threadIdx.x / 32, lane = threadIdx.x % 32;
  const float4* op = reinterpret_cast<const float4*>(p.opart + (int64_t)bh * p.nsplit * DK_D) + lane;
  const float4* lp = reinterpret_cast<const float4*>(p.lpart) + (int64_t)bh * p.nsplit;  // four parts per chunk
  float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  float l = 0.0f;
  int s = r;
  for (; s + 3 * CB_GROUPS < p.nsplit; s += 4 * CB_GROUPS) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = op[(int64_t)(s + u * CB_GROUPS) * (DK_D / 4)];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      o.x += v[u].x, o.y += v[u].y, o.z += v[u].z, o.w += v[u].w;
      if (lane == 0) {
        const float4 q = lp[s + u * CB_GROUPS];
        l += (q.x + q.y) + (q.z + q.w);
      }
    }
  }
  for (; s < p.nsplit; s += CB_GROUPS) {
    const float4 v = op[(int64_t)s * (DK_D / 4)];
    o.x += v.x, o.y += v.y, o.z += v.z, o.w += v.w;
    if (lane == 0) {
      const float4 q = lp[s];
      l += (q.x + q.y) + (q.z + q.w);
    }
  }
  osum[r][lane] = o;
  if (lane == 0) lsum[r] = l;
  __syncthreads();
  if (threadIdx.x < DK_D) {
    const int d = threadIdx.x;
    const float* os = reinterpret_cast<const float*>(osum);
    float v[CB_GROUPS];
#pragma unroll
    for (int g = 0; g < CB_GROUPS; ++g) v[g] = os[g * DK_D + d];
    float l[CB_GROUPS];
#pragma unroll
    for (int g = 0; g < CB_GROUPS; ++g) l[g] = lsum[g];
    // pairwise, in a fixed order
#pragma unroll
    for (int sp = 1; sp < CB_GROUPS; sp *= 2)
#pragma unroll
      for (int g = 0; g < CB_GROUPS; g += 2 * sp) v[g] += v[g + sp], l[g] += l[g + sp];
    const float on = v[0], ln = l[0];
    p.out[(int64_t)bh * DK_D + d] = on / ln;
  }
}

template <int MG>
int launch_scores(const DecodeArgs& a, int items, cudaStream_t st) {
  // K codes: [B*Hkv*Tmax rows][64 B], boxes of 256 keys with the 64-byte swizzle of the MMA operand
  CUtensorMap mk;
  if (int e = encode_tiled_2d(&mk, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.k_codes, DK_D / 2,
                              (uint64_t)a.B * a.Hkv * a.Tmax, DK_D / 2, DK_D / 2, DK_KEYS, CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  if (int e = set_smem_attr((const void*)decode_scores_kernel<MG>, (int)dsc::SMEM)) return e;
  // two CTAs per SM (shared memory allows no third), each holding 256 TMEM columns
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  decode_scores_kernel<MG><<<std::min(items, 2 * sms), dsc::THREADS, dsc::SMEM, st>>>(mk, a);
  return check_launch("decode_scores_kernel");
}

template <int MG>
int launch_pv(const DecodeArgs& a, int items, cudaStream_t st) {
  using C = dpv::Cfg<MG>;
  // codes: [B*Hkv*D rows][Tmax/2 bytes], tiles of 128 channels x 256 keys; group scales: [rows][Tmax/16]
  const uint64_t rows = (uint64_t)a.B * a.Hkv * DK_D;
  CUtensorMap mv, ms;
  if (int e = encode_tiled_2d(&mv, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.v_codes, (uint64_t)a.Tmax / 2, rows,
                              (uint64_t)a.Tmax / 2, DK_KEYS / 2, DK_D, CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  // without a group-scale prefix the map is never read; it then describes the per-element scales
  const uint8_t* s16 = a.v_scales16 ? a.v_scales16 : a.v_scales;
  if (int e = encode_tiled_2d(&ms, CU_TENSOR_MAP_DATA_TYPE_UINT8, s16, (uint64_t)a.Tmax / 16, rows,
                              (uint64_t)a.Tmax / 16, DK_KEYS / 16, DK_D, CU_TENSOR_MAP_SWIZZLE_NONE))
    return e;
  if (int e = set_smem_attr((const void*)decode_pv_kernel<MG>, (int)C::SMEM)) return e;
  // one CTA per SM: each holds all 512 TMEM columns
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  decode_pv_kernel<MG><<<std::min(items, sms), dpv::THREADS, C::SMEM, st>>>(mv, ms, a);
  return check_launch("decode_pv_kernel");
}

}  // namespace
}  // namespace fp4

using namespace fp4;

extern "C" int64_t fp4attn_decode_workspace_size(int B, int Hq, int len) {
  if (B <= 0 || Hq <= 0 || len <= 0) return -1;
  const int64_t nsplit = (len + DK_KEYS - 1) / DK_KEYS;
  const int64_t bh = (int64_t)B * Hq;
  return (bh * nsplit * DK_KEYS + bh * nsplit * (DK_D + 4) + bh) * (int64_t)sizeof(float);
}

extern "C" int fp4attn_decode_ex(const uint8_t* q_codes, const uint8_t* q_scales, const float* q_g,
                                 const uint8_t* k_codes, const uint8_t* k_scales, const float* k_g,
                                 const uint8_t* v_codes, const uint8_t* v_scales, const float* v_g,
                                 const uint8_t* v_scales16, int len16, int B, int Hq, int Hkv, int D, int len,
                                 int Tmax, float scaling, float* out, void* workspace, int64_t workspace_bytes,
                                 void* stream) {
  clear_error();
  if (len16 < 0 || len16 > len || len16 % 16 || (len16 > 0 && !v_scales16) || (uintptr_t)v_scales16 % 16)
    return set_error(FP4ATTN_ERR_ARG, "group-scale prefix: len16 a multiple of 16 in [0, len], 16-byte aligned");
  if (!q_codes || !q_scales || !q_g || !k_codes || !k_scales || !k_g || !v_codes || !v_scales || !v_g || !out ||
      !workspace)
    return set_error(FP4ATTN_ERR_ARG, "null pointer");
  if (D != DK_D) return set_error(FP4ATTN_ERR_UNSUPPORTED, "head_dim must be %d", DK_D);
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || len <= 0 || Tmax < len)
    return set_error(FP4ATTN_ERR_ARG, "bad shape");
  if (Tmax % DK_KEYS) return set_error(FP4ATTN_ERR_ARG, "Tmax must be a multiple of %d", DK_KEYS);
  if (Hq / Hkv > DK_MAXG) return set_error(FP4ATTN_ERR_UNSUPPORTED, "more than %d query heads per KV head", DK_MAXG);
  if (((uintptr_t)k_codes | (uintptr_t)v_codes | (uintptr_t)k_scales | (uintptr_t)v_scales | (uintptr_t)k_g |
       (uintptr_t)v_g | (uintptr_t)workspace) % 16)
    return set_error(FP4ATTN_ERR_ARG, "cache buffers and workspace must be 16-byte aligned");
  const int64_t need = fp4attn_decode_workspace_size(B, Hq, len);
  if (workspace_bytes < need) return set_error(FP4ATTN_ERR_ARG, "workspace of %lld bytes, %lld needed",
                                               (long long)workspace_bytes, (long long)need);
  const int nsplit = (len + DK_KEYS - 1) / DK_KEYS;
  const int64_t bh = (int64_t)B * Hq;
  float* S = static_cast<float*>(workspace);
  float* opart = S + bh * nsplit * DK_KEYS;
  float* lpart = opart + bh * nsplit * DK_D;
  unsigned int* mrow = reinterpret_cast<unsigned int*>(lpart + bh * nsplit * 4);
  DecodeArgs a{q_codes, q_scales, q_g,    k_codes, k_scales, k_g,  v_codes, v_scales,
               v_g,     v_scales16, B,   Hq,      Hkv,      len,  Tmax,    nsplit,
               len16 / DK_KEYS, scaling, S, opart, lpart, mrow, out};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(mrow, 0xFF, bh * sizeof(unsigned int), st) != cudaSuccess)
    return set_error(FP4ATTN_ERR_CUDA, "memset: %s", cudaGetErrorString(cudaGetLastError()));
  const int items = nsplit * B * Hkv;
  const int G = Hq / Hkv;
  if (int e = G <= 4 ? launch_scores<4>(a, items, st) : G <= 8 ? launch_scores<8>(a, items, st)
                                                          : launch_scores<16>(a, items, st))
    return e;
  const int e = G <= 4 ? launch_pv<4>(a, items, st) : G <= 8 ? launch_pv<8>(a, items, st) : launch_pv<16>(a, items, st);
  if (e) return e;
  decode_combine_kernel<<<(unsigned)bh, CB_GROUPS * 32, 0, st>>>(a);
  return check_launch("decode_combine_kernel");
}

extern "C" int fp4attn_decode(const uint8_t* q_codes, const uint8_t* q_scales, const float* q_g,
                              const uint8_t* k_codes, const uint8_t* k_scales, const float* k_g,
                              const uint8_t* v_codes, const uint8_t* v_scales, const float* v_g, int B, int Hq,
                              int Hkv, int D, int len, int Tmax, float scaling, float* out, void* workspace,
                              int64_t workspace_bytes, void* stream) {
  return fp4attn_decode_ex(q_codes, q_scales, q_g, k_codes, k_scales, k_g, v_codes, v_scales, v_g, nullptr, 0, B, Hq,
                           Hkv, D, len, Tmax, scaling, out, workspace, workspace_bytes, stream);
}
