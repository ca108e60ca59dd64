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
//      appended them, so a token's scale is per channel), per-token g_v [B][Tmax];
//      optionally the same scales once per 16-token group [B][Hkv][Tmax/16][D]
//      for a prefix of len16 tokens whose groups each came from one block (a
//      call that started on a group boundary with whole blocks per sequence).
//      Chunks of 256 keys inside that prefix read the 2 KB of group scales
//      instead of 32 KB of per-element scales.
// Tmax is a multiple of 256, so every chunk of 256 keys is whole in memory.
// The query comes in the same packed form (row mode on its [B, Hq*D] view):
// codes [B][Hq*D/2], E4M3 scales [B][Hq*D/16], g_q [B].
//
// Work item = (chunk of 256 keys, b, KV head).  Three kernels, HBM-bound:
//  * scores: persistent CTAs stream their items' K through a ring of shared
//    memory stages (one producer warp, bulk copies, mbarriers); eight warps
//    compute S = (code*scale)_q . (code*scale)_k * g_q * g_k * scaling on
//    mma.sync m16n8k16 (fp16 products exact, fp32 accumulate; the query heads
//    of the KV head are the MMA rows, 8 keys its columns), write S and fold
//    each row's maximum into an order-free atomic maximum;
//  * pv: the same ring over V and S; the exact row max, e = exp2((S - m)
//    log2 e), the NVFP4 fake-quant of e per 16 keys (as the prefill kernel
//    does), then O-partial^T = (code*scale)_v^T (P-hat * g_v)^T on mma.sync
//    m16n8k16 (V-hat exact in fp16; P-hat * g_v as fp16 hi + lo, since V's
//    per-token g_v is not exact in fp16), fp32 accumulate;
//  * combine: O = sum O-partial / sum l over the chunks, in a fixed order.
#include <stdint.h>

#include <algorithm>

#include "common.cuh"
#include "fp4attn.h"
#include "sm100.cuh"
#include "status.h"

namespace fp4 {

FP4_DEFINE_STATUS_READER(decode_status)

namespace {

constexpr int DK_KEYS = 256;  // keys per work item
constexpr int DK_MAXG = 16;   // query heads per KV head
constexpr int DK_D = 128;     // head dim
constexpr int DK_WARPS = 8;   // consumer warps (plus one producer warp)
constexpr int DK_THREADS = (DK_WARPS + 1) * 32;

// scores stage: K codes | K scales | g_k
constexpr uint32_t SC_KC = DK_KEYS * DK_D / 2;
constexpr uint32_t SC_KS = DK_KEYS * DK_D / 16;
constexpr uint32_t SC_KG = DK_KEYS * 4;
constexpr uint32_t SC_STAGE = SC_KC + SC_KS + SC_KG;
constexpr int SC_STAGES = 3;
// pv stage: V codes | V scales | g_v | S of the G heads
constexpr uint32_t PV_VC = DK_KEYS * DK_D / 2;
constexpr uint32_t PV_VS16 = DK_KEYS / 16 * DK_D;  // V scales of a chunk, one row per 16-token group
constexpr uint32_t PV_VG = DK_KEYS * 4;
constexpr uint32_t PV_S1 = DK_KEYS * 4;  // S of one head
// MG bounds the query heads per KV head (NT = MG/8 rounded up MMA n-tiles of
// 8 heads).  Dynamic shared memory: the ring, then P-hat * g_v * 2^E as fp16
// hi and lo rows [2*MG][PV_PH_LD] (keys in MMA k order), then each warp's
// partial O [DK_WARPS][MG][PV_PART_LD] (dim 16g + c at position c*8 + g).
constexpr int PV_PART_LD = 132;  // 4 mod 16 floats: the fragment stores hit 32 distinct banks
constexpr int PV_PH_LD = DK_KEYS + 8;  // fp16 P-hat row: 132 words, so the 8 heads of a B load hit 32 banks
// NW consumer warps: warp w owns KPW = 256 / NW keys of an item (KSTEPS MMA
// k-steps of 16); with 16 warps the two half-warps split the heads in phase e.
template <int MG, int NW>
struct PvCfg {
  static constexpr int NT = (MG + 7) / 8;
  static constexpr int KPW = DK_KEYS / NW;
  static constexpr int KSTEPS = KPW / 16;
  static constexpr int LG = 32 / KPW;  // lane groups sharing a key in phase e
  static constexpr int THREADS = (NW + 1) * 32;
  // 4 heads per KV head: three stages fit two CTAs on an SM
  static constexpr int STAGES = MG == 8 ? 4 : 3;
  static constexpr uint32_t STAGE = PV_VC + PV_VS16 + PV_VG + MG * PV_S1;
  static constexpr uint32_t RING = STAGES * STAGE;
  static constexpr uint32_t PH = 2 * MG * PV_PH_LD * 2;
  static constexpr uint32_t PART = NW * MG * PV_PART_LD * 4;
  static constexpr uint32_t SMEM = RING + PH + PART;
  static_assert(KPW == 16 || KPW == 32, "a warp covers one or two 16-key steps");
  static_assert(SMEM + 2048 <= 232448, "shared memory");
};

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
  float* lpart;        // [B*Hq][nsplit]
  unsigned int* mrow;  // [B*Hq] row maximum of S (float bits, atomic; 0xFFFFFFFF = none yet)
  float* out;          // [B][Hq][D]
};

__device__ __forceinline__ uint32_t cvt_e2m1x2_f16x2(uint32_t byte) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(r) : "r"(byte));
  return r;
}
__device__ __forceinline__ uint32_t cvt_e4m3x2_f16x2(uint32_t two_bytes) {
  uint32_t r;
  asm("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(r) : "r"(two_bytes));
  return r;
}
__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// order-preserving float maximum on the bit pattern (exact, order-free)
__device__ __forceinline__ void atomic_max_f32(unsigned int* a, float v) {
  if (!(v < 0.0f)) atomicMax(reinterpret_cast<int*>(a), __float_as_int(v));
  else atomicMin(a, __float_as_uint(v));
}
// named barrier 1 over the NW consumer warps (the producer warp is not in it)
template <int NW = DK_WARPS>
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"r"(NW * 32) : "memory"); }
// consumers_sync that also ANDs a flag over the consumer threads (every warp sees the same answer)
template <int NW = DK_WARPS>
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
// Lane (r, q) of a warp: key r of the warp's group of 8; the MMA's K index
// is permuted so that lane q's B values for chunk c (k = 2q, 2q+1, 2q+8,
// 2q+9) are dims 32q + 4c + 0..3: its code bytes of a key are one contiguous
// run (bytes 16q..16q+15) and its scales two bytes (2q, 2q+1).  The A
// fragment uses the same permutation, so the dot product is unchanged.
__global__ void __launch_bounds__(DK_THREADS) decode_scores_kernel(DecodeArgs p) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ __align__(8) uint64_t full[SC_STAGES], empty[SC_STAGES];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  int i0, i1;
  item_range(p.nsplit * p.B * p.Hkv, i0, i1);
  if (threadIdx.x == 0) {
    for (int s = 0; s < SC_STAGES; ++s) mbar_init(&full[s], 1), mbar_init(&empty[s], DK_WARPS);
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == DK_WARPS) {
    if (lane == 0)
      produce<SC_STAGES>(full, empty, ring, SC_STAGE, i0, i1, 0x401, [&](int item, uint8_t* st, uint64_t* bar) {
        const int bk = item / p.nsplit, split = item % p.nsplit, b = bk / p.Hkv;
        const int64_t row = (int64_t)bk * p.Tmax + (int64_t)split * DK_KEYS;
        mbar_arrive_expect_tx(bar, SC_STAGE);
        bulk_load(st, p.k_codes + row * (DK_D / 2), SC_KC, bar);
        bulk_load(st + SC_KC, p.k_scales + row * (DK_D / 16), SC_KS, bar);
        bulk_load(st + SC_KC + SC_KS, p.k_g + (int64_t)b * p.Tmax + (int64_t)split * DK_KEYS, SC_KG, bar);
      });
    return;
  }
  const int G = p.Hq / p.Hkv;
  const int r = lane / 4, q = lane % 4;
  const int ks = p.nsplit * DK_KEYS;
  int cur = -1;
  uint32_t afr[DK_D / 16][4];
  float gq = 0.0f;
  float mx[2] = {-INFINITY, -INFINITY};  // rows r, r+8
  auto flush = [&](int bk) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
    }
    const int64_t bh0 = (int64_t)(bk / p.Hkv) * p.Hq + (bk % p.Hkv) * G;
    if (q == 0) {
      if (r < G) atomic_max_f32(&p.mrow[bh0 + r], mx[0]);
      if (r + 8 < G) atomic_max_f32(&p.mrow[bh0 + r + 8], mx[1]);
    }
  };
  for (int it = 0; it < i1 - i0; ++it) {
    const int item = i0 + it, bk = item / p.nsplit, split = item % p.nsplit;
    const int b = bk / p.Hkv, hk = bk % p.Hkv;
    if (bk != cur) {
      if (cur >= 0) flush(cur);
      cur = bk;
      mx[0] = mx[1] = -INFINITY;
      gq = p.q_g[b];
      // A: rows r, r+8 (query heads); k = 2q,2q+1 -> dims 32q+4c+0,1; k = 2q+8,2q+9 -> dims 32q+4c+2,3
      const int64_t qel = ((int64_t)b * p.Hq + hk * G) * DK_D;
#pragma unroll
      for (int c = 0; c < DK_D / 16; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = r + (i & 1) * 8, dim = 32 * q + 4 * c + 2 * (i >> 1);
          uint32_t v = 0;
          if (row < G) {
            const int64_t el = qel + row * DK_D + dim;
            const uint32_t sb = p.q_scales[el / 16];
            v = hmul2u(cvt_e2m1x2_f16x2(p.q_codes[el / 2]), cvt_e4m3x2_f16x2(sb | (sb << 8)));
          }
          afr[c][i] = v;
        }
    }
    const int s = it % SC_STAGES;
    if (!mbar_wait(&full[s], (it / SC_STAGES) & 1, 0x402)) break;
    const uint8_t* st = ring + (size_t)s * SC_STAGE;
    const int64_t srow = ((int64_t)b * p.Hq + hk * G) * ks;
#pragma unroll
    for (int gi = 0; gi < DK_KEYS / 8 / DK_WARPS; ++gi) {
      const int kl = (warp + gi * DK_WARPS) * 8;  // first key of the group (in the item)
      const uint4 cw = *reinterpret_cast<const uint4*>(st + (kl + r) * (DK_D / 2) + 16 * q);
      const uint32_t sw = *reinterpret_cast<const uint16_t*>(st + SC_KC + (kl + r) * (DK_D / 16) + 2 * q);
      const float2 kg = *reinterpret_cast<const float2*>(st + SC_KC + SC_KS + (kl + 2 * q) * 4);
      const uint32_t s0 = cvt_e4m3x2_f16x2((sw & 0xFFu) * 0x101u), s1 = cvt_e4m3x2_f16x2((sw >> 8) * 0x101u);
      const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int c = 0; c < DK_D / 16; ++c) {
        // dims 32q + 4c + 0..3 = bytes 2c, 2c+1 of the lane's run (block 2q + c/4)
        const uint32_t w = words[c / 2] >> (16 * (c & 1));
        const uint32_t sc = c < 4 ? s0 : s1;
        mma16816(acc, afr[c], hmul2u(cvt_e2m1x2_f16x2(w & 0xFFu), sc),
                 hmul2u(cvt_e2m1x2_f16x2((w >> 8) & 0xFFu), sc));
      }
      // acc: rows r (0,1) and r+8 (2,3); keys kl + 2q, +1
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = r + (i >> 1) * 8, key = split * DK_KEYS + kl + 2 * q + (i & 1);
        if (row >= G) continue;
        float sv = -INFINITY;
        if (key < p.len) sv = __fmul_rn(__fmul_rn(__fmul_rn(acc[i], gq), (i & 1) ? kg.y : kg.x), p.scaling);
        p.S[srow + (int64_t)row * ks + key] = sv;
        mx[i >> 1] = fmaxf(mx[i >> 1], sv);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (cur >= 0) flush(cur);
}

// -------------------------------------------------------------------- pv
// Phase e: thread t handles key t of the item (e, the per-16-key NVFP4
// fake-quant of e, P-hat * g_v), as the prefill kernel quantizes P.
//
// PV on mma.sync m16n8k16 (fp16 operands, fp32 accumulate), transposed:
// O^T[dim][head] += V-hat^T[dim][key] * (P-hat g_v)^T[key][head].  Warp w owns
// keys 32w..32w+31 of the item -- the keys its own phase-e threads produced,
// so no CTA barrier sits between the phases -- as two k-steps of 16 keys.
//  * A = V-hat = code * scale, exact in fp16 (E2M1 x E4M3 has at most five
//    significant bits and lies in [2^-10, 2688]).  M index: m-tile mt, row g
//    (g = lane/4) is dim 16g + 2mt, row g+8 dim 16g + 2mt + 1, so a lane's
//    dims are one 8-byte run of codes and one 16-byte run of scales per key.
//  * K index within a k-step: k = 8h + 2t + j (t = lane%4) is key 8h + 4j + t,
//    so lane t's keys are t, t+4, t+8, t+12 and each load instruction reads
//    four consecutive key rows (no bank conflicts).  The code nibbles of keys
//    t and t+4 are merged into (key t, key t+4) bytes, which convert to the
//    A register pairs directly.
//  * B = P-hat * g_v as fp16 hi + lo (22 significant bits; g_v varies along
//    the keys, so it cannot be factored out), scaled by a per-warp power of
//    two 2^E that keeps the largest value below 2^15 (P-hat <= 1.03125 and
//    g_v < 2^(e+1)); the partial O is scaled back by 2^-E, exactly.
//  * N index: head 8nt + g (heads >= G are zero).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

template <int MG, int NW>
__global__ void __launch_bounds__((NW + 1) * 32) decode_pv_kernel(DecodeArgs p) {
  using C = PvCfg<MG, NW>;
  constexpr int NT = C::NT, KPW = C::KPW, LG = C::LG;
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ __align__(8) uint64_t full[C::STAGES], empty[C::STAGES];
  __shared__ float lred[NW][MG];
  __shared__ float rcp_tab[128];  // correctly rounded 1/s of every non-negative E4M3 scale byte (0 -> 0)
  __half(*ph)[PV_PH_LD] = reinterpret_cast<__half(*)[PV_PH_LD]>(ring + C::RING);  // hi rows [0,MG), lo rows [MG,2MG)
  float(*part)[MG][PV_PART_LD] = reinterpret_cast<float(*)[MG][PV_PART_LD]>(ring + C::RING + C::PH);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, t = threadIdx.x;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int G = p.Hq / p.Hkv;
  int i0, i1;
  item_range(p.nsplit * p.B * p.Hkv, i0, i1);
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) mbar_init(&full[s], 1), mbar_init(&empty[s], NW);
    fence_barrier_init();
  }
  if (threadIdx.x < 128) {
    const float sv = e4m3_to_f32((uint8_t)threadIdx.x);
    rcp_tab[threadIdx.x] = sv == 0.0f ? 0.0f : __frcp_rn(sv);
  }
  __syncthreads();
  if (warp == NW) {
    if (lane == 0)
      produce<C::STAGES>(full, empty, ring, C::STAGE, i0, i1, 0x411, [&](int item, uint8_t* st, uint64_t* bar) {
        const int bk = item / p.nsplit, split = item % p.nsplit, b = bk / p.Hkv, hk = bk % p.Hkv;
        const int64_t row = (int64_t)bk * p.Tmax + (int64_t)split * DK_KEYS;
        const int ks = p.nsplit * DK_KEYS;
        const bool compact = split < p.nsplit16;
        mbar_arrive_expect_tx(bar, PV_VC + (compact ? PV_VS16 : 0u) + PV_VG + (uint32_t)G * PV_S1);
        bulk_load(st, p.v_codes + row * (DK_D / 2), PV_VC, bar);
        if (compact) bulk_load(st + PV_VC, p.v_scales16 + row / 16 * DK_D, PV_VS16, bar);
        bulk_load(st + PV_VC + PV_VS16, p.v_g + (int64_t)b * p.Tmax + (int64_t)split * DK_KEYS, PV_VG, bar);
        for (int g = 0; g < G; ++g)
          bulk_load(st + PV_VC + PV_VS16 + PV_VG + g * PV_S1,
                    p.S + ((int64_t)b * p.Hq + hk * G + g) * ks + (int64_t)split * DK_KEYS, PV_S1, bar);
      });
    return;
  }
  const float log2e = 1.4426950408889634f, r6 = __frcp_rn(6.0f);
  // phase e: this lane's key (lane group lg takes heads lg, lg + LG, ...) and its MMA k position
  const int lg = lane / KPW;
  const int key = KPW * warp + lane % KPW;
  const int kr = key & 15;
  const int kpos = (key & ~15) + (kr & 8) + 2 * (kr & 3) + ((kr >> 2) & 1);
  int cur = -1;
  float m[MG];
#pragma unroll
  for (int g = 0; g < MG; ++g) m[g] = 0.0f;
  for (int it = 0; it < i1 - i0; ++it) {
    const int item = i0 + it, bk = item / p.nsplit, split = item % p.nsplit;
    const int b = bk / p.Hkv, hk = bk % p.Hkv;
    const int64_t bh0 = (int64_t)b * p.Hq + hk * G;
    if (bk != cur) {
      cur = bk;
#pragma unroll
      for (int g = 0; g < MG; ++g)
        if (g < G) m[g] = __uint_as_float(p.mrow[bh0 + g]);
    }
    const int s = it % C::STAGES;
    // a failed wait reads stale shared memory below; all consumers then leave together at consumers_all
    const bool landed = mbar_wait(&full[s], (it / C::STAGES) & 1, 0x412);
    uint8_t* st = ring + (size_t)s * C::STAGE;
    const int nlive = min(DK_KEYS, p.len - split * DK_KEYS);
    const bool live = key < nlive;
    // chunks inside the group-scale prefix hold every key live
    const bool compact = split < p.nsplit16;
    const int64_t vrow = (int64_t)bk * p.Tmax + (int64_t)split * DK_KEYS;  // first cache row of the chunk
    if (!live && lg == 0) {
      // the key is past len: whatever the cache holds there becomes V = 0 (its scales read as 0
      // below; P-hat is 0 there too)
      uint4* vc = reinterpret_cast<uint4*>(st + key * (DK_D / 2));
#pragma unroll
      for (int i = 0; i < DK_D / 2 / 16; ++i) vc[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    const float gv = live ? reinterpret_cast<const float*>(st + PV_VC + PV_VS16)[key] : 0.0f;
    float gmax = gv;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, o));
    // 2^E with P-hat * g_v * 2^E < 2^15 (P-hat <= 1.03125 < 2, g_v < 2^(e+1))
    int E = 0;
    if (gmax > 0.0f) E = max(-100, min(100, 13 - (((__float_as_int(gmax) >> 23) & 0xFF) - 127)));
    const float up = __int_as_float((E + 127) << 23), down = __int_as_float((127 - E) << 23);
    {
      const float* Ss = reinterpret_cast<const float*>(st + PV_VC + PV_VS16 + PV_VG);
#pragma unroll
      for (int gi = 0; gi < (MG + LG - 1) / LG; ++gi) {
        const int g = lg + gi * LG;
        if (gi * LG >= G) break;  // uniform over the warp
        const bool on = g < G;
        float mg = m[gi * LG];  // m[g] with compile-time indices (lg is 0 or 1)
        if constexpr (LG > 1) {
          if (gi * LG + 1 < MG && lg == 1) mg = m[gi * LG + 1];
        }
        const float e = live && on ? exp2f(__fmul_rn(Ss[min(g, G - 1) * DK_KEYS + key] - mg, log2e)) : 0.0f;
        float am = e;  // block of 16 keys = 16 consecutive lanes
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        const uint8_t sb = e4m3_satfinite(__fmul_rn(am, r6));  // e >= 0: sb < 0x80
        const float sf = e4m3_to_f32(sb);
        const float rs = rcp_tab[sb & 0x7F];
        const uint32_t byte = e2m1x2(__fmaf_rn(e, rs, 0.0f), 0.0f);
        const float code = __half2float(__ushort_as_half((unsigned short)(cvt_e2m1x2_f16x2(byte) & 0xFFFFu)));
        const float x = live ? __fmul_rn(__fmul_rn(__fmul_rn(code, sf), gv), up) : 0.0f;
        const __half hi = __float2half_rn(x);
        if (on) {
          ph[g][kpos] = hi;
          ph[MG + g][kpos] = __float2half_rn(x - __half2float(hi));
        }
        float l = e;
#pragma unroll
        for (int o = KPW / 2; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (on && lane % KPW == 0) lred[warp][g] = l;
      }
    }
    __syncwarp();
    float acc[NT][8][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int mt = 0; mt < 8; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nt][mt][i] = 0.0f;
#pragma unroll
    for (int kstep = 0; kstep < C::KSTEPS; ++kstep) {
      const int kb = KPW * warp + 16 * kstep;
      uint2 cw[4];
      uint4 sw[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int kk = kb + t4 + 4 * i;
        cw[i] = *reinterpret_cast<const uint2*>(st + kk * (DK_D / 2) + 8 * g8);
      }
      if (compact) {
        // the four keys of this lane lie in one 16-token group: one row of group scales
        const uint4 s16 = *reinterpret_cast<const uint4*>(st + PV_VC + (kb >> 4) * DK_D + 16 * g8);
#pragma unroll
        for (int i = 0; i < 4; ++i) sw[i] = s16;
      } else {
        // per-element scales straight from the cache (L2): only the chunks past the prefix
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int kk = kb + t4 + 4 * i;
          sw[i] = kk < nlive ? __ldg(reinterpret_cast<const uint4*>(p.v_scales + (vrow + kk) * DK_D + 16 * g8))
                             : make_uint4(0u, 0u, 0u, 0u);
        }
      }
      uint32_t bhi[NT][2], blo[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int h = 8 * nt + g8;
        const bool on = h < G;
        bhi[nt][0] = on ? *reinterpret_cast<const uint32_t*>(&ph[h][kb + 2 * t4]) : 0u;
        bhi[nt][1] = on ? *reinterpret_cast<const uint32_t*>(&ph[h][kb + 2 * t4 + 8]) : 0u;
        blo[nt][0] = on ? *reinterpret_cast<const uint32_t*>(&ph[MG + h][kb + 2 * t4]) : 0u;
        blo[nt][1] = on ? *reinterpret_cast<const uint32_t*>(&ph[MG + h][kb + 2 * t4 + 8]) : 0u;
      }
      // code bytes of key pairs (t, t+4) and (t+8, t+12): even dims in E, odd dims in O,
      // the first key of the pair in the low nibble
      uint32_t ev[2][2], od[2][2];
#pragma unroll
      for (int pr = 0; pr < 2; ++pr)
#pragma unroll
        for (int wd = 0; wd < 2; ++wd) {
          const uint32_t x = wd ? cw[2 * pr].y : cw[2 * pr].x, y = wd ? cw[2 * pr + 1].y : cw[2 * pr + 1].x;
          ev[pr][wd] = (x & 0x0F0F0F0Fu) | ((y << 4) & 0xF0F0F0F0u);
          od[pr][wd] = ((x >> 4) & 0x0F0F0F0Fu) | (y & 0xF0F0F0F0u);
        }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int wd = mt >> 2, sh = 8 * (mt & 3);
        const uint32_t sel = (mt & 1) ? 0x7362u : 0x5140u;
        uint32_t a[4];
#pragma unroll
        for (int pr = 0; pr < 2; ++pr) {
          const uint32_t sx = (mt >> 1) == 0 ? sw[2 * pr].x : (mt >> 1) == 1 ? sw[2 * pr].y
                            : (mt >> 1) == 2 ? sw[2 * pr].z : sw[2 * pr].w;
          const uint32_t sy = (mt >> 1) == 0 ? sw[2 * pr + 1].x : (mt >> 1) == 1 ? sw[2 * pr + 1].y
                            : (mt >> 1) == 2 ? sw[2 * pr + 1].z : sw[2 * pr + 1].w;
          const uint32_t sc = prmt(sx, sy, sel);  // {s_x, s_y} of dim 2mt (low half), of dim 2mt+1 (high half)
          a[2 * pr] = hmul2u(cvt_e2m1x2_f16x2((ev[pr][wd] >> sh) & 0xFFu), cvt_e4m3x2_f16x2(sc & 0xFFFFu));
          a[2 * pr + 1] = hmul2u(cvt_e2m1x2_f16x2((od[pr][wd] >> sh) & 0xFFu), cvt_e4m3x2_f16x2(sc >> 16));
        }
        // fragment order: a0 rows g / k 0-7, a1 rows g+8 / k 0-7, a2 rows g / k 8-15, a3 rows g+8 / k 8-15
        const uint32_t fr[4] = {a[0], a[1], a[2], a[3]};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma16816(acc[nt][mt], fr, bhi[nt][0], bhi[nt][1]);
          mma16816(acc[nt][mt], fr, blo[nt][0], blo[nt][1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp's V rows and scores are no longer read
    // acc[nt][mt]: (dim 16g+2mt, head 8nt+2t), (dim, head+1), (dim+1, head), (dim+1, head+1)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int h = 8 * nt + 2 * t4, c = 2 * mt;
        if (h < G) {
          part[warp][h][c * 8 + g8] = acc[nt][mt][0] * down;
          part[warp][h][(c + 1) * 8 + g8] = acc[nt][mt][2] * down;
        }
        if (h + 1 < G) {
          part[warp][h + 1][c * 8 + g8] = acc[nt][mt][1] * down;
          part[warp][h + 1][(c + 1) * 8 + g8] = acc[nt][mt][3] * down;
        }
      }
    if (!consumers_all<NW>(landed)) break;  // part and lred are complete
    if (t < G) {
      float l = 0.0f;
      for (int w = 0; w < NW; ++w) l += lred[w][t];
      p.lpart[(bh0 + t) * p.nsplit + split] = l;
    }
    for (int i = t; i < G * DK_D; i += NW * 32) {
      // consecutive threads read consecutive positions (no bank conflicts); pos c*8 + g holds dim 16g + c
      const int g = i / DK_D, pos = i % DK_D, d = 16 * (pos & 7) + (pos >> 3);
      float v[NW];
#pragma unroll
      for (int w = 0; w < NW; ++w) v[w] = part[w][g][pos];
      // pairwise sums in a fixed order: ((w0 + w1) + (w2 + w3)) + ...
#pragma unroll
      for (int sp = 1; sp < NW; sp *= 2)
#pragma unroll
        for (int w = 0; w < NW; w += 2 * sp) v[w] += v[w + sp];
      p.opart[((bh0 + g) * p.nsplit + split) * DK_D + d] = v[0];
    }
    consumers_sync<NW>();  // part and lred are rewritten by the next item
  }
}

// O = sum over chunks of O-partial / sum of l.  One CTA per (b, query head):
// group r of 32 threads sums chunks r, r + 8, r + 16, ... (4 dims per thread,
// 16-byte loads, every load of the group issued before the adds), then the
// eight group sums are added in a fixed order.
constexpr int CB_GROUPS = 8;
__global__ void __launch_bounds__(CB_GROUPS * 32) decode_combine_kernel(DecodeArgs p) {
  __shared__ float4 osum[CB_GROUPS][DK_D / 4];
  __shared__ float lsum[CB_GROUPS];
  const int bh = blockIdx.x, r = threadIdx.x / 32, lane = threadIdx.x % 32;
  const float4* op = reinterpret_cast<const float4*>(p.opart + (int64_t)bh * p.nsplit * DK_D) + lane;
  const float* lp = p.lpart + (int64_t)bh * p.nsplit;
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
      if (lane == 0) l += lp[s + u * CB_GROUPS];
    }
  }
  for (; s < p.nsplit; s += CB_GROUPS) {
    const float4 v = op[(int64_t)s * (DK_D / 4)];
    o.x += v.x, o.y += v.y, o.z += v.z, o.w += v.w;
    if (lane == 0) l += lp[s];
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
    const float on = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    const float ln = ((lsum[0] + lsum[1]) + (lsum[2] + lsum[3])) + ((lsum[4] + lsum[5]) + (lsum[6] + lsum[7]));
    p.out[(int64_t)bh * DK_D + d] = on / ln;
  }
}

// Persistent grid: as many CTAs as are resident at once, at most one per item.
int persistent_grid(const void* fn, uint32_t smem, int items, int threads = DK_THREADS) {
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem) != cudaSuccess || per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  return std::min(items, sms * per_sm);
}

template <int MG, int NW>
int launch_pv(const DecodeArgs& a, int items, cudaStream_t st) {
  using C = PvCfg<MG, NW>;
  if (int e = set_smem_attr((const void*)decode_pv_kernel<MG, NW>, (int)C::SMEM)) return e;
  const int grid = persistent_grid((const void*)decode_pv_kernel<MG, NW>, C::SMEM, items, C::THREADS);
  decode_pv_kernel<MG, NW><<<grid, C::THREADS, C::SMEM, st>>>(a);
  return check_launch("decode_pv_kernel");
}

}  // namespace
}  // namespace fp4

using namespace fp4;

extern "C" int64_t fp4attn_decode_workspace_size(int B, int Hq, int len) {
  if (B <= 0 || Hq <= 0 || len <= 0) return -1;
  const int64_t nsplit = (len + DK_KEYS - 1) / DK_KEYS;
  const int64_t bh = (int64_t)B * Hq;
  return (bh * nsplit * DK_KEYS + bh * nsplit * (DK_D + 1) + bh) * (int64_t)sizeof(float);
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
  unsigned int* mrow = reinterpret_cast<unsigned int*>(lpart + bh * nsplit);
  DecodeArgs a{q_codes, q_scales, q_g,    k_codes, k_scales, k_g,  v_codes, v_scales,
               v_g,     v_scales16, B,   Hq,      Hkv,      len,  Tmax,    nsplit,
               len16 / DK_KEYS, scaling, S, opart, lpart, mrow, out};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(mrow, 0xFF, bh * sizeof(unsigned int), st) != cudaSuccess)
    return set_error(FP4ATTN_ERR_CUDA, "memset: %s", cudaGetErrorString(cudaGetLastError()));
  const int items = nsplit * B * Hkv;
  constexpr uint32_t sc_smem = SC_STAGES * SC_STAGE;
  if (int e = set_smem_attr((const void*)decode_scores_kernel, (int)sc_smem)) return e;
  decode_scores_kernel<<<persistent_grid((const void*)decode_scores_kernel, sc_smem, items), DK_THREADS, sc_smem,
                         st>>>(a);
  if (int e = check_launch("decode_scores_kernel")) return e;
  const int G = Hq / Hkv;
  // eight consumer warps for every group size (sixteen, with the heads split between half-warps in
  // phase e, measured 199 us against 175 us at B 8 / 32768 keys / 4 heads per KV head)
  const int e = G <= 4 ? launch_pv<4, 8>(a, items, st)
                : G <= 8 ? launch_pv<8, 8>(a, items, st) : launch_pv<16, 8>(a, items, st);
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
