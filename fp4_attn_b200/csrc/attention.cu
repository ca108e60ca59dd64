// attention.cu -- NVFP4 attention forward on sm_100a (tcgen05 + TMA + TMEM).
//
// Computes what the reference's patched attention computes
// (llama_patch.py:57-105 after the Q/K/V fake-quant of llama_patch.py:167-196):
//
//   S = (Qhat Khat^T) * scaling (+ causal mask);  P = softmax(S)
//   Phat = NVFP4 fake-quant of P, per query row (row global scale = row max
//          of P, blocks of 16 along keys)              (llama_patch.py:81-99)
//   O = Phat Vhat                                       (llama_patch.py:102)
//
// with Qhat/Khat NVFP4 along head_dim under a per-token global scale and
// Vhat NVFP4 along tokens under a per-token global scale
// (single_nvfp4(v2d.T, global_scale_aligned=False), llama_patch.py:196).
//
// Numerics.  P's block scales depend on P relative to the row maximum, so
// each 128-query tile runs two passes over its keys: pass 1 computes S with
// FP4 tensor-core MMAs and keeps the exact row maximum; pass 2 recomputes S,
// forms e = exp2((S - max) * log2 e) (the reference's P / rowmax(P)), sums
// e for the softmax denominator, quantizes e to E2M1 codes with an E4M3
// scale per 16 keys exactly as the reference's quantizer does, and writes
// Phat = code * scale (exact in fp16) into TMEM.  The reference's per-token
// V global scale varies along PV's reduction axis, so PV cannot use
// block-scaled FP4 without changing the result; Vhat is prepared once as
// two fp16 planes (hi + lo, 22 significant bits, fp4attn_prepare_v) and PV
// runs as two kind::f16 MMAs with A = Phat read from TMEM.  O = acc / sum.
//
// Schedule.  A work unit is (batch, query head, 128-query tile); persistent
// CTAs take units longest-first in snake order (causal cost grows with the tile index).
// Warp 0 loads Q and K by TMA (codes, scale atoms, global scales), warp 2
// loads V-hat tiles, warp 1 issues the QK^T MMAs, warp 3 the PV MMAs, and
// warps 4-19 are four softmax warpgroups: warpgroup q owns key columns 32q..32q+31 of every
// tile.  S is double-buffered in TMEM, so QK(j+2) runs as soon as every softmax
// warp has loaded S(j); P-hat has its own TMEM buffer, freed by PV's commit.
// Every wait is bounded (sm100.cuh).
#include <cuda.h>
#include <cuda_bf16.h>

#include <stdlib.h>

#include <type_traits>

#include "common.cuh"
#include "attn_softmax.cuh"
#include "attn_internal.h"
#include "fp4attn.h"
#include "sm100.cuh"
#include "status.h"
#include "tmap.h"

namespace fp4 {

FP4_DEFINE_STATUS_READER(attn_status)

namespace attn {
constexpr int BM = 128, BN = 128, HD = 128;
#ifndef FP4ATTN_K_STAGES
#define FP4ATTN_K_STAGES 4
#endif
constexpr int NK = FP4ATTN_K_STAGES;  // K stages (codes + scale atoms + g)
constexpr int NV = 2;   // V-hat stages, one 128-key tile each (hi and lo planes)
constexpr int NWG = 4;  // softmax warpgroups; warpgroup q owns key columns 32q .. 32q+31
constexpr int THREADS = 128 + NWG * 128;
// shared memory map (bytes, all pieces 1024-aligned where TMA/UMMA need it)
constexpr int Q_BYTES = BM * HD / 2;  // 8 KB of E2M1 codes
constexpr int OFF_Q = 0, OFF_QSF = 8192, OFF_GQ = 9216;
// second (residual) Q slice of dual-slice Q: codes, scale atoms, g
constexpr int OFF_QLO = 10240, OFF_QLOSF = 18432, OFF_GQLO = 19456;
constexpr int K_STAGE = 10240;  // codes 8 KB, scale atoms 1 KB, gk 512 B
constexpr int OFF_K = 20480;
constexpr int V_HALF = HD * 64 * 2;  // 128 rows (d) x 64 keys x fp16 = one plane of a half tile (one TMA box)
constexpr int V_STAGE = 4 * V_HALF;  // keys 0-63 hi, lo; keys 64-127 hi, lo
constexpr int OFF_V = OFF_K + NK * K_STAGE;
constexpr int OFF_STAT = OFF_V + NV * V_STAGE;  // m[NWG][128], l[NWG][128], residual max[NWG][128]
constexpr int OFF_RCP = OFF_STAT + 3 * NWG * 128 * 4;
constexpr int OFF_MROW = OFF_RCP + 128 * 4;  // the unit's 128 row maxima (PRE), loaded with Q
constexpr int OFF_BAR = OFF_MROW + 128 * 4;
constexpr int SMEM_BYTES = OFF_BAR + 512 + 1024;
constexpr uint32_t TMEM_COLS = 512;
// TMEM columns: S0, S1, O, P (fp16, single-buffered; warpgroup q writes columns
// 16q..16q+15), Q scale atoms, K scale atoms per stage, the residual Q
// slice's scale atoms (456 + 8 * (NK + 1) of 512 columns).  With dual-slice Q, S0 and S1
// hold the two slices' products of the same key tile (S single-buffered).
constexpr uint32_t T_S = 0, T_O = 256, T_P = 384, T_SFA = 448, T_SFB = 456, T_SFA_LO = T_SFB + 8 * NK;
static_assert(T_SFA_LO + 8 <= TMEM_COLS, "K scale atoms of every stage must fit in TMEM");
static_assert(SMEM_BYTES <= 232448, "shared memory map exceeds the 227 KB a CTA can have");
}  // namespace attn

struct AttnArgs {
  const uint8_t* qsf;  // tcgen05 atoms, nkb4q = Hq*2 groups per 128-row block
  const float* gq;     // [B*Tp]
  const uint8_t* qsf_lo;  // residual Q slice (dual-slice Q), same layouts
  const float* gq_lo;
  const uint8_t* ksf;
  const float* gk;
  void* out;    // [B, T, Hq, HD], fp32 or (out_bf16) bf16
  int out_bf16;
  int B, Hq, Hkv, T, Tp;  // Hq / Hkv: the heads attended (and written to out)
  // The packed operands may hold more heads than are attended (a rank of a sharded job
  // quantizes whole batch rows): the attended heads start at head hq0 / hk0 of operands
  // with nkb4q / nkb4k scale atoms per 128-row block (2 per head) and HkvT KV heads.
  int hq0, hk0, nkb4q, nkb4k, HkvT, HqT;
  // Row maxima of z = (Q K^T) * gk per (batch, query head of the operands, row):
  // [B][HqT][Tp] fp32, written by fp4_rowmax_t_kernel and read by the attention kernels
  // instantiated with PRE (which then has no max pass of its own).
  float* row_max;
  // PV uses V-hat's lo plane only for query tiles qt < pv_lo_tiles (the hi plane is
  // V-hat rounded once to fp16); a large value keeps PV exact everywhere.
  int pv_lo_tiles;
  int causal;
  float scale_log2;  // scaling * log2(e)
  int units;
  long long* trace;  // optional event timeline (fp4attn_set_trace), [grid][kTraceSlots]
};

// Timeline slots recorded for each CTA's first work unit when tracing is on.
constexpr int kTraceSlots = 512;
enum TraceSlot {
  TR_QK = 0,        // + pass*32 + j : MMA issued QK (after its waits)
  TR_PV = 64,       // + j : MMA issued PV
  TR_PWAIT = 96,    // + j : MMA starts waiting for P
  TR_SFULL = 128,   // + pass*32 + j : softmax saw S ready
  TR_PDONE = 192,   // + j : softmax finished P (pass 2)
  TR_MDONE = 224,   // + j : softmax finished the tile (pass 1)
  TR_UNIT = 256,    // MMA saw Q ready
  TR_OFULL = 257,   // epilogue saw O ready
  TR_OFREE = 258,   // epilogue released O
  TR_UEND = 259,    // MMA committed the unit
  TR_START = 260,   // kernel start (after setup)
  TR_LDDONE = 288,  // + j : pass-2 scores in registers (warpgroup 0)
  TR_COMP = 320,    // + j : pass-2 Phat computed (warpgroup 0)
  TR_PDONE3 = 384,  // + j : softmax warpgroup 3 finished P (pass 2)
};

__device__ __forceinline__ void trace(const AttnArgs& p, uint32_t uc, int slot, int j) {
  if (p.trace && uc == 0 && j < 32 && slot + j < kTraceSlots)
    p.trace[(int64_t)blockIdx.x * kTraceSlots + slot + j] = (long long)clock64();
}

struct Unit {
  int qt, b, h;
};

__device__ __forceinline__ Unit unit_of(int u, const AttnArgs& p) {
  const int nqt = p.Tp / attn::BM;
  const int bh = p.B * p.Hq;
  Unit r;
  r.qt = nqt - 1 - u / bh;  // longest (latest) query tiles first
  const int x = u % bh;
  r.b = x / p.Hq;
  r.h = x % p.Hq;
  return r;
}

// The i-th unit of this CTA, or -1 past its last.  Units are numbered longest
// first; round r hands them to CTAs 0..G-1 on even rounds and G-1..0 on odd
// rounds ("snake"), which evens out the causal cost across CTAs (only the
// last round is partial, so a CTA's units are rounds 0, 1, ... without gaps).
__device__ __forceinline__ int cta_unit(int i, int units) {
  const int G = (int)gridDim.x, c = (int)blockIdx.x;
  const int u = i * G + ((i & 1) ? G - 1 - c : c);
  return u < units ? u : -1;
}

__device__ __forceinline__ int kv_tiles(const Unit& un, const AttnArgs& p) {
  return p.causal ? un.qt + 1 : p.Tp / attn::BN;
}

// TRACE: record the event timeline (fp4attn_set_trace); the plain instantiation
// has no trace code at all.  DQ: dual-slice Q (a second, residual Q slice;
// both QK products of a key tile go to the two S accumulators and combine per
// row).  DP: dual-slice P (a residual pass between the max pass and the PV
// pass finds each row's residual scale; the PV pass writes hi + lo).  PRE: the
// row maxima come from fp4_rowmax_t_kernel (p.row_max, loaded with Q), so the
// kernel has no max pass and reads each K tile once (single-slice Q only).
template <bool TRACE, bool DQ, bool DP, bool PRE>
__global__ void __launch_bounds__(attn::THREADS, 1)
    fp4_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmQlo,
                    const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmVhi,
                    const __grid_constant__ CUtensorMap tmVlo, AttnArgs p) {
  using namespace attn;
  static_assert(!(PRE && DQ), "precomputed row maxima are for single-slice Q");
  constexpr int NPASS = (DP ? 3 : 2) - (PRE ? 1 : 0);  // QK passes per unit; the last one feeds PV
  // With a single pass the PV thread releases each K stage for the softmax warps: it
  // waits for all of them to finish P (after their last read of the stage's gk) anyway.
  constexpr bool PV_RELEASES_K = NPASS == 1;
  // SPLIT (the precomputed-maximum kernel): one S buffer and two P buffers, so the softmax
  // stores P(j+1) while PV(j) still runs; S is read at the start of a tile, so QK(j+1) lands
  // while the softmax still works on tile j.  Otherwise two S buffers (the max pass has
  // little work to hide QK's latency behind) and one P buffer.  TMEM: S [0,128), O
  // [128,256), P0, P1 [256,384), scale atoms from 384 (SPLIT).
  constexpr bool SPLIT = PRE;
  constexpr uint32_t tO = SPLIT ? 128 : T_O, tP = SPLIT ? 256 : T_P;
  constexpr uint32_t tSFA = SPLIT ? 384 : T_SFA, tSFB = SPLIT ? 392 : T_SFB;
  static_assert(!SPLIT || tSFB + 8 * NK <= TMEM_COLS, "TMEM columns of the split layout");
  constexpr int oK = OFF_K, oV = OFF_V, oSTAT = OFF_STAT, oRCP = OFF_RCP, oMROW = OFF_MROW;
  constexpr int oBAR = OFF_BAR;
  constexpr int nV = NV;
  auto tr = [&](uint32_t uc, int slot, int j) {
    if constexpr (TRACE) trace(p, uc, slot, j);
  };
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* stat_m = reinterpret_cast<float*>(sm + oSTAT);
  float* stat_l = stat_m + NWG * 128;
  float* stat_r = stat_m + 2 * NWG * 128;
  float* rcp = reinterpret_cast<float*>(sm + oRCP);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + oBAR);
  uint64_t* q_full = bar + 0;
  uint64_t* q_empty = bar + 1;
  uint64_t* k_full = bar + 2;          // [NK]
  uint64_t* k_empty = k_full + NK;     // [NK]
  uint64_t* v_full = k_empty + NK;     // [NV]
  uint64_t* v_empty = v_full + NV;     // [NV]
  uint64_t* s_full = v_empty + NV;     // [2] S buffer written (MMA commit)
  uint64_t* s_free = s_full + 2;       // [2] S buffer read by every softmax warp
  uint64_t* p_full = s_free + 2;       // [2] P written by every softmax warp
  uint64_t* p_free = p_full + 2;       // [2] PV has read P (PV thread's commit)
  uint64_t* o_full = p_free + 2;
  uint64_t* o_free = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 1);
  static_assert(2 + 2 * NK + 2 * NV + 10 + 1 <= 64, "barriers exceed their 512-byte slot");

  const int warp = threadIdx.x / 32;
  const int nkb4q = p.nkb4q, nkb4k = p.nkb4k;
  const int group = p.Hq / p.Hkv;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1 + 4 * NWG);  // MMA commit + every softmax warp (they read g and m)
    for (int i = 0; i < NK; ++i) {
      mbar_init(&k_full[i], 1);
      // MMA commit + every softmax warp (they read gk), or + the PV thread for them
      mbar_init(&k_empty[i], PV_RELEASES_K ? 2 : 1 + 4 * NWG);
    }
    for (int i = 0; i < nV; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4 * NWG);  // every softmax warp has loaded its rows
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], 4 * NWG);  // every softmax warp has stored its P
      mbar_init(&p_free[i], 1);
    }
    mbar_init(o_full, 1);
    mbar_init(o_free, 1);
    fence_barrier_init();
  }
  if (threadIdx.x < 128) {
    // correctly rounded 1/s for every non-negative E4M3 scale byte (0 -> 0, get_reciprocal)
    const float s = e4m3_to_f32((uint8_t)threadIdx.x);
    rcp[threadIdx.x] = s == 0.0f ? 0.0f : __frcp_rn(s);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) tr(0, TR_START, 0);

  if (warp == 0) {
    // ------------------------------------------------- producer: Q and K
    if (elect_one_lane()) {
      tma_prefetch_desc(&tmQ);
      if constexpr (DQ) tma_prefetch_desc(&tmQlo);
      tma_prefetch_desc(&tmK);
      uint32_t kc = 0, uc = 0;
      for (int i = 0, u = cta_unit(0, p.units); u >= 0; u = cta_unit(++i, p.units), ++uc) {
        const Unit un = unit_of(u, p);
        const int n = kv_tiles(un, p);
        const int hq = p.hq0 + un.h, hk = p.hk0 + un.h / group;  // heads within the operands
        const int qrow = un.b * p.Tp + un.qt * BM;
        if (uc > 0) mbar_wait(q_empty, (uc - 1) & 1, 0x201);
        mbar_arrive_expect_tx(q_full, (DQ ? 2 : 1) * (Q_BYTES + 1024 + 512) + (PRE ? 512 : 0));
        tma_load_2d(sm + OFF_Q, &tmQ, q_full, hq * (HD / 2), qrow);
        if constexpr (PRE)
          bulk_load(sm + oMROW, p.row_max + ((int64_t)un.b * p.HqT + hq) * p.Tp + un.qt * BM, 512, q_full);
        bulk_load(sm + OFF_QSF, p.qsf + ((int64_t)(qrow / 128) * nkb4q + 2 * hq) * 512, 1024, q_full);
        bulk_load(sm + OFF_GQ, p.gq + qrow, 512, q_full);
        if constexpr (DQ) {
          tma_load_2d(sm + OFF_QLO, &tmQlo, q_full, hq * (HD / 2), qrow);
          bulk_load(sm + OFF_QLOSF, p.qsf_lo + ((int64_t)(qrow / 128) * nkb4q + 2 * hq) * 512, 1024, q_full);
          bulk_load(sm + OFF_GQLO, p.gq_lo + qrow, 512, q_full);
        }
        for (int pass = 0; pass < NPASS; ++pass) {
          for (int j = 0; j < n; ++j, ++kc) {
            const int s = kc % NK;
            if (kc >= NK) mbar_wait(&k_empty[s], ((kc / NK) - 1) & 1, 0x202);
            uint8_t* ks = sm + oK + s * K_STAGE;
            const int krow = un.b * p.Tp + j * BN;
            mbar_arrive_expect_tx(&k_full[s], 8192 + 1024 + 512);
            tma_load_2d(ks, &tmK, &k_full[s], hk * (HD / 2), krow);
            bulk_load(ks + 8192, p.ksf + ((int64_t)(krow / 128) * nkb4k + 2 * hk) * 512, 1024, &k_full[s]);
            bulk_load(ks + 9216, p.gk + krow, 512, &k_full[s]);
          }
        }
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------- producer: V-hat tiles (pass 2)
    if (elect_one_lane()) {
      tma_prefetch_desc(&tmVhi);
      tma_prefetch_desc(&tmVlo);
      uint32_t vc = 0;
      for (int i = 0, u = cta_unit(0, p.units); u >= 0; u = cta_unit(++i, p.units)) {
        const Unit un = unit_of(u, p);
        const int n = kv_tiles(un, p);
        const int vrow = (un.b * p.HkvT + p.hk0 + un.h / group) * HD;
        for (int j = 0; j < n; ++j) {
          const bool lo = un.qt < p.pv_lo_tiles;  // the lo plane only where PV reads it
          const int vs = vc % nV;
          if (vc >= nV) mbar_wait(&v_empty[vs], ((vc / nV) - 1) & 1, 0x203);
          uint8_t* v = sm + oV + vs * V_STAGE;
          mbar_arrive_expect_tx(&v_full[vs], lo ? V_STAGE : V_STAGE / 2);
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            tma_load_2d(v + 2 * half * V_HALF, &tmVhi, &v_full[vs], j * BN + 64 * half, vrow);
            if (lo) tma_load_2d(v + (2 * half + 1) * V_HALF, &tmVlo, &v_full[vs], j * BN + 64 * half, vrow);
          }
          ++vc;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- QK^T issue
    // One elected thread issues every S = Q K^T (both passes) into the two S
    // buffers; a buffer is reused once every softmax warp has loaded the
    // scores in it (s_free).
    if (elect_one_lane()) {
      const uint32_t idq = idesc_nvf4(BM, BN);
      uint32_t kc = 0, uc = 0;
      uint32_t suse0 = 0, suse1 = 0;  // QKs issued into each S buffer (scalars, not an indexed array)
      auto issue_qk = [&](int j, int kb, int pass) {
        const uint32_t su = kb ? suse1 : suse0;
        if (su > 0) mbar_wait(&s_free[kb], (su - 1) & 1, 0x211);
        const int s = kc % NK;
        mbar_wait(&k_full[s], (kc / NK) & 1, 0x212);
        tc_fence_after();
        if (pass < 2) tr(uc, TR_QK + 32 * pass, j);
        uint8_t* ks = sm + oK + s * K_STAGE;
        const uint32_t sfb = tmem + tSFB + 8 * s;
        tmem_cp_sf_atom(sfb, smem_desc(smem_u32(ks + 8192), 16, 128, kSwizzleNone));
        tmem_cp_sf_atom(sfb + 4, smem_desc(smem_u32(ks + 8192 + 512), 16, 128, kSwizzleNone));
        const uint32_t d = tmem + T_S + 128 * kb;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const uint64_t ad = smem_desc(smem_u32(sm + OFF_Q) + kk * 32, 16, 512, kSwizzle64B);
          const uint64_t bd = smem_desc(smem_u32(ks) + kk * 32, 16, 512, kSwizzle64B);
          mma_nvf4(d, ad, bd, idq, tmem + tSFA + 4 * kk, sfb + 4 * kk, kk > 0 ? 1u : 0u);
        }
        if constexpr (DQ) {  // residual slice into the second accumulator
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const uint64_t ad = smem_desc(smem_u32(sm + OFF_QLO) + kk * 32, 16, 512, kSwizzle64B);
            const uint64_t bd = smem_desc(smem_u32(ks) + kk * 32, 16, 512, kSwizzle64B);
            mma_nvf4(tmem + T_S + 128, ad, bd, idq, tmem + T_SFA_LO + 4 * kk, sfb + 4 * kk, kk > 0 ? 1u : 0u);
          }
        }
        tc_commit(&k_empty[s]);
        tc_commit(&s_full[kb]);
        if (kb) ++suse1;
        else ++suse0;
        ++kc;
      };
      for (int i = 0, u = cta_unit(0, p.units); u >= 0; u = cta_unit(++i, p.units), ++uc) {
        const Unit un = unit_of(u, p);
        const int n = kv_tiles(un, p);
        mbar_wait(q_full, uc & 1, 0x213);
        tr(uc, TR_UNIT, 0);
        tc_fence_after();
        tmem_cp_sf_atom(tmem + tSFA, smem_desc(smem_u32(sm + OFF_QSF), 16, 128, kSwizzleNone));
        tmem_cp_sf_atom(tmem + tSFA + 4, smem_desc(smem_u32(sm + OFF_QSF + 512), 16, 128, kSwizzleNone));
        if constexpr (DQ) {
          tmem_cp_sf_atom(tmem + T_SFA_LO, smem_desc(smem_u32(sm + OFF_QLOSF), 16, 128, kSwizzleNone));
          tmem_cp_sf_atom(tmem + T_SFA_LO + 4, smem_desc(smem_u32(sm + OFF_QLOSF + 512), 16, 128, kSwizzleNone));
        }
        for (int pass = 0; pass < NPASS; ++pass)
          for (int j = 0; j < n; ++j) issue_qk(j, (DQ || SPLIT) ? 0 : (j & 1), pass);
        tc_commit(q_empty);
        tr(uc, TR_UEND, 0);
      }
    }
  } else if (warp == 3) {
    // --------------------------------------------------------- PV issue
    // One elected thread issues O += P V-hat (hi and lo planes) per pass-2
    // tile once every softmax warp has written its rows of P and the V-hat
    // tile has landed; its commit frees the P buffer for the next tile.
    if (elect_one_lane()) {
      const uint32_t idv = idesc_f16(BM, HD);
      uint32_t vc = 0, uc = 0, pu = 0, tcnt = 0;
      for (int i = 0, u = cta_unit(0, p.units); u >= 0; u = cta_unit(++i, p.units), ++uc) {
        const Unit un = unit_of(u, p);
        const int n = kv_tiles(un, p);
        const int parts = un.qt < p.pv_lo_tiles ? 2 : 1;  // hi + lo planes, or hi alone
        for (int j = 0; j < n; ++j, ++tcnt) {
          const int pb = SPLIT ? (int)(pu & 1) : 0;
          mbar_wait(&v_full[vc % nV], (vc / nV) & 1, 0x215);  // the tile's (hi) stage
          tr(uc, TR_PWAIT, j);
          mbar_wait(&p_full[pb], (SPLIT ? (pu >> 1) : pu) & 1, 0x214);
          ++pu;
          if constexpr (PV_RELEASES_K) mbar_arrive(&k_empty[tcnt % NK]);
          if (j == 0 && uc > 0) mbar_wait(o_free, (uc - 1) & 1, 0x216);
          tc_fence_after();
          tr(uc, TR_PV, j);
          {
            const int vs = vc % nV;
            const uint32_t v = smem_u32(sm + oV + vs * V_STAGE);
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk) {  // keys 16kk .. 16kk+15
              const uint32_t a = tmem + tP + 64 * pb + 8 * kk;  // fp16 P of keys 16kk..16kk+15
              for (int part = 0; part < parts; ++part) {  // hi, lo planes
                const uint32_t vb = v + ((kk >> 2) * 2 + part) * V_HALF + (kk & 3) * 32;
                mma_f16_ts(tmem + tO, a, smem_desc(vb, 16, 1024, kSwizzle128B), idv,
                           (j > 0 || kk > 0 || part > 0) ? 1u : 0u);
              }
            }
            tc_commit(&v_empty[vs]);
            ++vc;
          }
          tc_commit(&p_free[pb]);
        }
        tc_commit(o_full);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------- softmax warpgroups
    // Every warpgroup works on every key tile: warpgroup q owns key columns
    // 32q .. 32q+31 (its quarter of S, its quarter of P).
    const int q = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + (threadIdx.x & 31);  // row of the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float r6 = __frcp_rn(6.0f);
    const bool leader = threadIdx.x % 128 == 0;
    const bool wlead = (threadIdx.x & 31) == 0;  // lane 0 arrives on behalf of its warp
    const int col0 = 32 * q;
    uint32_t kc = 0, uc = 0, pt = 0;
    uint32_t sfu0 = 0, sfu1 = 0;  // completions seen per S buffer
    // ---- epilogue of a finished unit: O rows / l, columns 32q .. 32q+31, then O is free
    bool pend = false;
    uint32_t pend_uc = 0;
    float pend_rl = 0.0f;
    int64_t pend_off = -1;  // element offset of this thread's 32 outputs, -1 for rows past T
    auto epilogue = [&]() {
      mbar_wait(o_full, pend_uc & 1, 0x224);
      if (threadIdx.x == 128) tr(pend_uc, TR_OFULL, 0);
      tc_fence_after();
      uint32_t a[32];
      tmem_ld32(tmem + lane_base + tO + col0, a);
      tmem_ld_wait();
      if (pend_off >= 0) {
        if (p.out_bf16) {  // rounded to bf16 as the reference's bf16 matmul output is
          uint4* d4 = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + pend_off);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(a[8 * i + 2 * k]) * pend_rl,
                                                             __uint_as_float(a[8 * i + 2 * k + 1]) * pend_rl);
              w[k] = *reinterpret_cast<const uint32_t*>(&h);
            }
            d4[i] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        } else {
          float4* d4 = reinterpret_cast<float4*>(static_cast<float*>(p.out) + pend_off);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            d4[i] = make_float4(__uint_as_float(a[4 * i]) * pend_rl, __uint_as_float(a[4 * i + 1]) * pend_rl,
                                __uint_as_float(a[4 * i + 2]) * pend_rl, __uint_as_float(a[4 * i + 3]) * pend_rl);
        }
      }
      tc_fence_before();
      named_bar(1 + NWG, NWG * 128);
      if (threadIdx.x == 128) {
        mbar_arrive(o_free);
        tr(pend_uc, TR_OFREE, 0);
      }
      pend = false;
    };
    for (int i = 0, u = cta_unit(0, p.units); u >= 0; u = cta_unit(++i, p.units), ++uc) {
      const Unit un = unit_of(u, p);
      const int n = kv_tiles(un, p);
      const int qpos = un.qt * BM + r;  // query index within the sequence
      mbar_wait(q_full, uc & 1, 0x221);
      const float ghi = reinterpret_cast<const float*>(sm + OFF_GQ)[r];
      const float uscale = ghi * p.scale_log2;
      // dual-slice Q: acc = acc_hi + acc_lo * (g_lo / g_hi), so the row keeps u = g_hi * scaling * log2 e
      float ratio = 0.0f;
      if constexpr (DQ) {
        const float glo = reinterpret_cast<const float*>(sm + OFF_GQLO)[r];
        ratio = ghi == 0.0f ? 0.0f : __fdiv_rn(glo, ghi);
      }
      const uint64_t ratio2 = pk2(ratio, ratio);
      float m = -INFINITY;
      if constexpr (PRE) m = reinterpret_cast<const float*>(sm + oMROW)[r];
      // g (and m) are in registers: this warp no longer needs the unit's Q buffer
      __syncwarp();
      if (wlead) mbar_arrive(q_empty);
      auto load_s = [&](int kb, uint32_t(&a)[32]) {
        tmem_ld32(tmem + lane_base + T_S + 128 * kb + col0, a);
        if constexpr (DQ) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // the residual slice's scores, 16 columns at a time
            uint32_t b[16];
            tmem_ld16(tmem + lane_base + T_S + 128 + col0 + 16 * h, b);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
              float x0, x1;
              upk2(fma2(pk2(__uint_as_float(b[i]), __uint_as_float(b[i + 1])), ratio2,
                        pk2(__uint_as_float(a[16 * h + i]), __uint_as_float(a[16 * h + i + 1]))),
                   x0, x1);
              a[16 * h + i] = __float_as_uint(x0);
              a[16 * h + i + 1] = __float_as_uint(x1);
            }
          }
        } else {
          tmem_ld_wait();
        }
      };
      // ---- pass 1: row maximum of z = acc * gk over this quarter's keys
      if constexpr (!PRE) {
      for (int j = 0; j < n; ++j, ++kc) {
        const int kb = (DQ || SPLIT) ? 0 : (j & 1), s = kc % NK;
        mbar_wait(&s_full[kb], (kb ? sfu1 : sfu0) & 1, 0x222);
        if (kb) ++sfu1;
        else ++sfu0;
        if (leader && q == 0) tr(uc, TR_SFULL, j);
        tc_fence_after();
        uint32_t a[32];
        load_s(kb, a);
        // every warp releases what it has read on its own (no warpgroup barrier)
        tc_fence_before();
        __syncwarp();
        if (wlead) mbar_arrive(&s_free[kb]);
        const uint32_t gk = smem_u32(sm + oK + s * K_STAGE + 9216) + 4 * col0;
        // keys with column > lim are masked (causal diagonal tile, or keys past T)
        const int lim = (p.causal && j == un.qt) ? r : (p.T - 1 - j * BN);
        if (lim < col0 + 31) m = chunk_max<true>(a, gk, col0, lim, m);
        else m = chunk_max<false>(a, gk, col0, lim, m);
        __syncwarp();
        if (wlead) mbar_arrive(&k_empty[s]);
        if (leader && q == 0) tr(uc, TR_MDONE, j);
      }
      stat_m[q * 128 + r] = m;
      named_bar(1 + NWG, NWG * 128);
#pragma unroll
      for (int w = 0; w < NWG; ++w) m = fmaxf(m, stat_m[w * 128 + r]);
      }
      const float mu = m == -INFINITY ? 0.0f : m * uscale;
      const uint64_t u2 = pk2(uscale, uscale), nmu2 = pk2(-mu, -mu);
      // ---- dual-slice P: residual pass, row max of |e - hi| over this quarter's keys
      float gr = 0.0f, rg = 0.0f;
      if constexpr (DP) {
        float rm = 0.0f;
        for (int j = 0; j < n; ++j, ++kc) {
          const int kb = (DQ || SPLIT) ? 0 : (j & 1), s = kc % NK;
          mbar_wait(&s_full[kb], (kb ? sfu1 : sfu0) & 1, 0x226);
          if (kb) ++sfu1;
          else ++sfu0;
          tc_fence_after();
          uint32_t a[32];
          load_s(kb, a);
          tc_fence_before();
          __syncwarp();
          if (wlead) mbar_arrive(&s_free[kb]);
          const uint32_t gk = smem_u32(sm + oK + s * K_STAGE + 9216) + 4 * col0;
          const int lim = (p.causal && j == un.qt) ? r : (p.T - 1 - j * BN);
          if (lim < col0 + 31) rm = chunk_rmax<true>(a, gk, col0, lim, u2, nmu2, smem_u32(rcp), r6, rm);
          else rm = chunk_rmax<false>(a, gk, col0, lim, u2, nmu2, smem_u32(rcp), r6, rm);
          __syncwarp();
          if (wlead) mbar_arrive(&k_empty[s]);
        }
        stat_r[q * 128 + r] = rm;
        named_bar(1 + NWG, NWG * 128);
#pragma unroll
        for (int w = 0; w < NWG; ++w) rm = fmaxf(rm, stat_r[w * 128 + r]);
        gr = rm;
        rg = rm == 0.0f ? 0.0f : __frcp_rn(rm);
      }
      // ---- pass 2: e = exp2(z*u - m*u), sum, NVFP4 fake-quant of e -> P quarter q
      uint64_t lsum2[4] = {pk2(0.0f, 0.0f), pk2(0.0f, 0.0f), pk2(0.0f, 0.0f), pk2(0.0f, 0.0f)};
      for (int j = 0; j < n; ++j, ++kc) {
        const int kb = (DQ || SPLIT) ? 0 : (j & 1), s = kc % NK;
        mbar_wait(&s_full[kb], (kb ? sfu1 : sfu0) & 1, 0x223);
        if (kb) ++sfu1;
        else ++sfu0;
        if (leader && q == 0) tr(uc, TR_SFULL + 32, j);
        tc_fence_after();
        uint32_t a[32];
        load_s(kb, a);
        // this warp's scores are in registers: release its share of the S buffer now
        tc_fence_before();
        __syncwarp();
        if (wlead) mbar_arrive(&s_free[kb]);
        if (leader && q == 0) tr(uc, TR_LDDONE, j);
        const uint32_t gk = smem_u32(sm + oK + s * K_STAGE + 9216) + 4 * col0;
        const int lim = (p.causal && j == un.qt) ? r : (p.T - 1 - j * BN);
        uint32_t pk[16];
        if constexpr (DP) {
          if (lim < col0 + 31) chunk_p_dual<true>(a, gk, col0, lim, u2, nmu2, smem_u32(rcp), r6, rg, gr, lsum2, pk);
          else chunk_p_dual<false>(a, gk, col0, lim, u2, nmu2, smem_u32(rcp), r6, rg, gr, lsum2, pk);
        } else {
          if (lim < col0 + 31) chunk_p<true>(a, gk, col0, lim, u2, nmu2, r6, lsum2, pk);
          else chunk_p<false>(a, gk, col0, lim, u2, nmu2, r6, lsum2, pk);
        }
        if (leader && q == 0) tr(uc, TR_COMP, j);
        // the previous unit's O is written while its last PV finishes, after this unit's
        // first P is computed; that also frees the accumulator for this unit's first PV
        if (j == 0 && pend) epilogue();
        // the previous tile's PV must have read P before quarter q is overwritten
        const int pb = SPLIT ? (int)(pt & 1) : 0;
        if constexpr (SPLIT) {
          if (pt >= 2) mbar_wait(&p_free[pb], ((pt >> 1) - 1) & 1, 0x225);
        } else {
          if (pt > 0) mbar_wait(&p_free[0], (pt - 1) & 1, 0x225);
        }
        tc_fence_after();
        tmem_st16(tmem + lane_base + tP + 64 * pb + 16 * q, pk);
        tmem_st_wait();
        tc_fence_before();
        ++pt;
        __syncwarp();
        if (wlead) {
          mbar_arrive(&p_full[pb]);
          if constexpr (!PV_RELEASES_K) mbar_arrive(&k_empty[s]);
        }
        if (leader && q == 0) tr(uc, TR_PDONE, j);
        if (leader && q == 3) tr(uc, TR_PDONE3, j);
      }
      float l0, l1;
      upk2(add2(add2(lsum2[0], lsum2[1]), add2(lsum2[2], lsum2[3])), l0, l1);
      stat_l[q * 128 + r] = l0 + l1;
      named_bar(1 + NWG, NWG * 128);
      float l = 0.0f;
#pragma unroll
      for (int w = 0; w < NWG; ++w) l += stat_l[w * 128 + r];
      // this unit's O is written after the next unit's pass 1 (or after the last unit)
      pend = true;
      pend_uc = uc;
      pend_rl = 1.0f / l;
      pend_off = qpos < p.T ? (((int64_t)un.b * p.T + qpos) * p.Hq + un.h) * HD + col0 : -1;
    }
    if (pend) epilogue();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

#include "attn_pingpong.cuh"
#include "attn_rowmax.cuh"

// ------------------------------------------------------------ V preparation
// Vhat = single_nvfp4(v2d.T, global_scale_aligned=False) in fp32 arithmetic
// (fp4_quant_utils.py:112-172 column mode on the [Hkv*D, B*T] view), written
// as two fp16 planes hi = fp16(Vhat), lo = fp16(Vhat - hi) in the layout the
// attention kernel loads: row (b*Hkv + h)*D + d, column t (Tp columns).
// One CTA per 16 consecutive tokens of the flattened B*T axis (one NVFP4
// block along tokens for every channel); the 16 x Hkv*D slab stays in
// shared memory in the input's own type (exact), so Hkv*D is limited by it.
// One CTA per 16 consecutive tokens of the flattened B*T axis (one NVFP4 block
// along tokens for every channel).  A thread owns channel pairs (2c, 2c+1) of
// one head (D is even) and reads their 16 token values as 16 two-element loads
// (consecutive pairs are consecutive addresses); sweep 2 reads them again (from
// L1: keeping them across the reduction costs more in spills).  Sweep 1
// takes the per-token max |v| on packed pairs in the input type (exact), a
// 16-shuffle transpose-reduce and a shared-memory pass finish it over the CTA;
// sweep 2 quantizes each channel's block of 16 tokens.
constexpr int VP_THREADS = 512;  // two CTAs per SM
constexpr int VP_MAX_HD_16 = 6144;  // bf16 / fp16 inputs
constexpr int VP_MAX_HD_32 = 3072;  // fp32 inputs

struct VPrepArgs {
  const void* v;  // bf16 / f16 / f32, [B, Hkv, T, D] with element strides
  int in_dtype;
  int64_t sB, sH, sT;
  int B, Hkv, T, D, Tp;
  __half* hi;
  __half* lo;
  float* vhat;  // optional fp32 Vhat, same layout
  float* g;     // optional per-token global scale [B*T]
  int vec;      // channel pairs are aligned words (even D and strides, aligned base): one load per pair
};

// fp16 pair -> two floats
__device__ __forceinline__ float2 vp_h2f(uint32_t h) { return __half22float2(*reinterpret_cast<const __half2*>(&h)); }

// Two channels' values: 16-bit inputs as one packed 32-bit word, fp32 as a float2.
template <int DT>
struct VPair {
  using W = typename std::conditional<DT == FP4_DT_F32, float2, uint32_t>::type;
  static __device__ __forceinline__ float2 f(W w) {
    if constexpr (DT == FP4_DT_F32) {
      return w;
    } else {
      using T = typename In<DT>::T;
      const T* e = reinterpret_cast<const T*>(&w);
      return make_float2(In<DT>::f(e[0]), In<DT>::f(e[1]));
    }
  }
  // per-lane max(|a|, |b|), NaN winning, in the input type (exact)
  static __device__ __forceinline__ W absmax(W a, W b) {
    if constexpr (DT == FP4_DT_F32) {
      return make_float2(nanmax(fabsf(a.x), fabsf(b.x)), nanmax(fabsf(a.y), fabsf(b.y)));
    } else {
      uint32_t r;
      if constexpr (DT == FP4_DT_BF16)
        asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a & 0x7FFF7FFFu), "r"(b & 0x7FFF7FFFu));
      else
        asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a & 0x7FFF7FFFu), "r"(b & 0x7FFF7FFFu));
      return r;
    }
  }
  static __device__ __forceinline__ W zero() {
    if constexpr (DT == FP4_DT_F32) return make_float2(0.0f, 0.0f);
    else return 0u;
  }
};

// One channel pair at q (q[0], q[1]): a single load when the pair is an aligned word.
template <int DT>
__device__ __forceinline__ typename VPair<DT>::W vp_pair(const typename In<DT>::T* q, bool vec) {
  using W = typename VPair<DT>::W;
  if (vec) return *reinterpret_cast<const W*>(q);
  if constexpr (DT == FP4_DT_F32) {
    return make_float2(q[0], q[1]);
  } else {
    const uint16_t* u = reinterpret_cast<const uint16_t*>(q);
    return (uint32_t)u[0] | ((uint32_t)u[1] << 16);
  }
}

// The 16 token values of the channel pair starting at c (zeros past B*T: the
// reference pads B*T to x16).  D is even, so a pair never straddles two heads.
template <int DT>
__device__ __forceinline__ void vp_load2(const VPrepArgs& p, int64_t j0, int c, typename VPair<DT>::W (&w)[16]) {
  using T = typename In<DT>::T;
  using W = typename VPair<DT>::W;
  const bool vec = p.vec != 0;
  const int h = c / p.D, d = c - h * p.D;
  const T* base = reinterpret_cast<const T*>(p.v) + (int64_t)h * p.sH + d;
  const int64_t BT = (int64_t)p.B * p.T;
  const int b0 = (int)(j0 / p.T), t0 = (int)(j0 - (int64_t)b0 * p.T);
  if (j0 + 16 <= BT && t0 + 16 <= p.T) {  // one batch row: a fixed token stride
    const T* q = base + (int64_t)b0 * p.sB + (int64_t)t0 * p.sT;
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = vp_pair<DT>(q + (int64_t)i * p.sT, vec);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int64_t jj = j0 + i;
      W x = VPair<DT>::zero();
      if (jj < BT) {
        const int b = (int)(jj / p.T), t = (int)(jj - (int64_t)b * p.T);
        x = vp_pair<DT>(base + (int64_t)b * p.sB + (int64_t)t * p.sT, vec);
      }
      w[i] = x;
    }
  }
}

// NVFP4 block of 16 tokens of channel e of the pair values w -> fp16 hi/lo words
// of token pairs; with VHAT the fp32 Vhat values too.  x * recip(g) is formed
// twice (for the block max, then for the codes) instead of being kept.
template <int DT, bool VHAT>
__device__ __forceinline__ void vp_quant16(const typename VPair<DT>::W (&w)[16], int e, const float* gtok,
                                           const float* rgtok, float r6, uint32_t (&hi2)[8], uint32_t (&lo2)[8],
                                           float* vh) {
  auto xs = [&](int i) {  // tokens i, i+1 of channel e, times recip(g) of each token
    const float2 a = VPair<DT>::f(w[i]), b = VPair<DT>::f(w[i + 1]);
    return __fmul2_rn(make_float2(e ? a.y : a.x, e ? b.y : b.x), make_float2(rgtok[i], rgtok[i + 1]));
  };
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; i += 4) {
    const float2 t0 = xs(i), t1 = xs(i + 2);
    amax = nanmax(amax, nanmax(absmax3(t0.x, t0.y, t1.x), fabsf(t1.y)));
  }
  const uint8_t sb = e4m3_torch(mul<FP4_ARITH_F32>(amax, r6));
  const float rs = recip<FP4_ARITH_F32>(e4m3_to_f32(sb));
  const bool nan_block = (sb & 0x7F) == 0x7F;
  uint32_t s2;  // the scale as an fp16 pair (exact: E4M3 values are fp16 values)
  asm("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(s2) : "r"((uint32_t)sb * 0x101u));
  const float2 rs2 = make_float2(rs, rs), zero2 = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    // x * recip(s) + 0 (one rounding; + 0 turns -0.0 into +0.0 like torch.sign), E2M1 RNE of tokens i, i+1
    const float2 a = __ffma2_rn(xs(i), rs2, zero2);
    uint32_t cs;  // (code * s) of both tokens as fp16: exact (|code * s| <= 6 * 448)
    asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
        : "=r"(cs)
        : "f"(a.x), "f"(a.y));
    if (nan_block) cs = 0u;
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(cs) : "r"(s2));
    const float2 q = __fmul2_rn(vp_h2f(cs), make_float2(gtok[i], gtok[i + 1]));  // (code * s) * g
    if constexpr (VHAT) {
      vh[i] = q.x;
      vh[i + 1] = q.y;
    }
    // hi = fp16(Vhat), lo = fp16(Vhat - hi)
    uint32_t hw, lw;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(hw) : "f"(q.y), "f"(q.x));
    const float2 hf = vp_h2f(hw);
    const float2 r = __fadd2_rn(q, make_float2(-hf.x, -hf.y));  // exactly q - hf
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(lw) : "f"(r.y), "f"(r.x));
    hi2[i / 2] = hw;
    lo2[i / 2] = lw;
  }
}

// VHAT: also write the fp32 Vhat.
template <int DT, bool VHAT>
__global__ void __launch_bounds__(VP_THREADS, 2) vprep_kernel(VPrepArgs p) {
  using W = typename VPair<DT>::W;
  __shared__ float red[VP_THREADS / 32][16];
  __shared__ float gtok[16], rgtok[16];
  const int HDn = p.Hkv * p.D;
  const int64_t BT = (int64_t)p.B * p.T;
  const int64_t j0 = (int64_t)blockIdx.x * 16;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // ---- sweep 1: per-token max |v| over this thread's channel pairs (packed, exact)
  W w[16];
  W mw[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) mw[i] = VPair<DT>::zero();
  for (int c = 2 * threadIdx.x; c < HDn; c += 2 * VP_THREADS) {
    vp_load2<DT>(p, j0, c, w);
#pragma unroll
    for (int i = 0; i < 16; ++i) mw[i] = VPair<DT>::absmax(mw[i], w[i]);
  }
  float m[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float2 t = VPair<DT>::f(mw[i]);
    m[i] = nanmax(t.x, t.y);
  }
  // transpose-reduce over the warp: after offsets 16, 8, 4, 2 a lane keeps one token's
  // partial max (token bits from lane bits 4..1), offset 1 completes it
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const bool up = lane & 16;
    const float keep = up ? m[k + 8] : m[k], send = up ? m[k] : m[k + 8];
    m[k] = nanmax(keep, __shfl_xor_sync(0xffffffffu, send, 16));
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const bool up = lane & 8;
    const float keep = up ? m[k + 4] : m[k], send = up ? m[k] : m[k + 4];
    m[k] = nanmax(keep, __shfl_xor_sync(0xffffffffu, send, 8));
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const bool up = lane & 4;
    const float keep = up ? m[k + 2] : m[k], send = up ? m[k] : m[k + 2];
    m[k] = nanmax(keep, __shfl_xor_sync(0xffffffffu, send, 4));
  }
  {
    const bool up = lane & 2;
    const float keep = up ? m[1] : m[0], send = up ? m[0] : m[1];
    m[0] = nanmax(keep, __shfl_xor_sync(0xffffffffu, send, 2));
  }
  m[0] = nanmax(m[0], __shfl_xor_sync(0xffffffffu, m[0], 1));
  if ((lane & 1) == 0) {
    const int tok = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
    red[warp][tok] = m[0];
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    float mx = 0.0f;
    for (int wi = 0; wi < VP_THREADS / 32; ++wi) mx = nanmax(mx, red[wi][threadIdx.x]);
    // per-token global scale: colmax of v2d.T * recip(1536) (fp4_quant_utils.py:136,139)
    const float g = mul<FP4_ARITH_F32>(mx, recip<FP4_ARITH_F32>(1536.0f));
    gtok[threadIdx.x] = g;
    rgtok[threadIdx.x] = recip<FP4_ARITH_F32>(g);
    if (p.g && j0 + threadIdx.x < BT) p.g[j0 + threadIdx.x] = g;
  }
  __syncthreads();
  // ---- sweep 2: NVFP4 block of 16 tokens per channel -> Vhat -> fp16 hi/lo planes
  const float r6 = recip<FP4_ARITH_F32>(6.0f);
  const int b0 = (int)(j0 / p.T), t0 = (int)(j0 - (int64_t)b0 * p.T);
  const bool fast_store = j0 + 16 <= BT && t0 + 16 <= p.T && t0 % 8 == 0 && p.Tp % 8 == 0;
  for (int c = 2 * threadIdx.x; c < HDn; c += 2 * VP_THREADS) {
    vp_load2<DT>(p, j0, c, w);
    const int h = c / p.D, d = c - h * p.D;
#pragma unroll
    for (int e = 0; e < 2; ++e) {  // the pair's two channels
      float vh[VHAT ? 16 : 1];
      uint32_t hi2[8], lo2[8];
      vp_quant16<DT, VHAT>(w, e, gtok, rgtok, r6, hi2, lo2, vh);
      const int de = d + e;
      if (fast_store) {
        // 16 tokens of one batch, contiguous in the output row: 16-byte stores
        const int64_t o = ((int64_t)(b0 * p.Hkv + h) * p.D + de) * p.Tp + t0;
        uint4* h4 = reinterpret_cast<uint4*>(p.hi + o);
        uint4* l4 = reinterpret_cast<uint4*>(p.lo + o);
        h4[0] = make_uint4(hi2[0], hi2[1], hi2[2], hi2[3]);
        h4[1] = make_uint4(hi2[4], hi2[5], hi2[6], hi2[7]);
        l4[0] = make_uint4(lo2[0], lo2[1], lo2[2], lo2[3]);
        l4[1] = make_uint4(lo2[4], lo2[5], lo2[6], lo2[7]);
        if constexpr (VHAT) {
#pragma unroll
          for (int i = 0; i < 16; ++i) p.vhat[o + i] = vh[i];
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int64_t jj = j0 + i;
          if (jj >= BT) continue;
          const int b = (int)(jj / p.T), t = (int)(jj - (int64_t)b * p.T);
          const int64_t oo = ((int64_t)(b * p.Hkv + h) * p.D + de) * p.Tp + t;
          const uint32_t hw = hi2[i / 2] >> (16 * (i & 1)), lw = lo2[i / 2] >> (16 * (i & 1));
          p.hi[oo] = __ushort_as_half((unsigned short)(hw & 0xFFFFu));
          p.lo[oo] = __ushort_as_half((unsigned short)(lw & 0xFFFFu));
          if constexpr (VHAT) p.vhat[oo] = vh[i];
        }
      }
    }
  }
}

template <int DT>
static void vprep_launch(const VPrepArgs& a, unsigned blocks, cudaStream_t st) {
  if (a.vhat) vprep_kernel<DT, true><<<blocks, VP_THREADS, 0, st>>>(a);
  else vprep_kernel<DT, false><<<blocks, VP_THREADS, 0, st>>>(a);
}

static int launch_vprep(const VPrepArgs& a, cudaStream_t st) {
  const unsigned blocks = (unsigned)(((int64_t)a.B * a.T + 15) / 16);
  switch (a.in_dtype) {
    case FP4_DT_F32: vprep_launch<FP4_DT_F32>(a, blocks, st); break;
    case FP4_DT_BF16: vprep_launch<FP4_DT_BF16>(a, blocks, st); break;
    case FP4_DT_F16: vprep_launch<FP4_DT_F16>(a, blocks, st); break;
    default: return set_error(FP4ATTN_ERR_ARG, "bad dtype");
  }
  return check_launch("vprep_kernel");
}

}  // namespace fp4

using namespace fp4;

static long long* g_trace = nullptr;

// Profiling aid: when buf is non-null, the next fp4attn_fwd_packed calls
// write an event timeline (SM clock cycles, clock64) of each CTA's first work unit into
// buf[cta * 512 + slot]; buf needs grid * 512 int64 entries.
extern "C" void fp4attn_set_trace(long long* buf) { g_trace = buf; }

extern "C" int fp4attn_prepare_v(const void* v, int in_dtype, int B, int Hkv, int T, int D, int64_t sB, int64_t sH,
                                 int64_t sT, int Tp, uint16_t* v_hi, uint16_t* v_lo, float* vhat, float* g,
                                 void* stream) {
  clear_error();
  if (!v || !v_hi || !v_lo) return set_error(FP4ATTN_ERR_ARG, "null pointer");
  if (B <= 0 || Hkv <= 0 || T <= 0 || D <= 0 || Tp < T) return set_error(FP4ATTN_ERR_ARG, "bad shape");
  const int max_hd = in_dtype == FP4_DT_F32 ? VP_MAX_HD_32 : VP_MAX_HD_16;
  if (Hkv * D > max_hd) return set_error(FP4ATTN_ERR_UNSUPPORTED, "Hkv*D > %d", max_hd);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (Tp > T) {  // padded key columns must read as zeros
    const size_t bytes = (size_t)B * Hkv * D * Tp * 2;
    if (cudaMemsetAsync(v_hi, 0, bytes, st) != cudaSuccess || cudaMemsetAsync(v_lo, 0, bytes, st) != cudaSuccess)
      return set_error(FP4ATTN_ERR_CUDA, "memset");
  }
  if (D % 2) return set_error(FP4ATTN_ERR_UNSUPPORTED, "head_dim must be even");
  const int esz = in_dtype == FP4_DT_F32 ? 4 : 2;
  const int vec = ((uintptr_t)v % (2 * esz) == 0) && sB % 2 == 0 && sH % 2 == 0 && sT % 2 == 0;
  VPrepArgs a{v, in_dtype, sB, sH, sT, B, Hkv, T, D, Tp, reinterpret_cast<__half*>(v_hi),
              reinterpret_cast<__half*>(v_lo), vhat, g, vec};
  return launch_vprep(a, st);
}

// Kernel-variant switches, read from the environment once per process: unset or
// anything but "0" means on.
static bool env_on(const char* name) {
  const char* e = getenv(name);
  return !(e && e[0] == '0');
}
// The single-slice attention (precomputed maxima, single-slice P) runs on the two-group
// kernel unless FP4ATTN_PINGPONG=0 selects the one-group kernel.
static bool pingpong_enabled() {
  static const bool on = env_on("FP4ATTN_PINGPONG");
  return on;
}

int fp4::launch_attention(const AttnLaunch& L, cudaStream_t st) {
  using namespace attn;
  const int B = L.B, HqT = L.HqT, HkvT = L.HkvT, T = L.T, Tp = L.Tp;
  if (L.D != HD) return set_error(FP4ATTN_ERR_UNSUPPORTED, "head_dim must be %d", HD);
  if (B <= 0 || HqT <= 0 || HkvT <= 0 || T <= 0 || HqT % HkvT != 0) return set_error(FP4ATTN_ERR_ARG, "bad shape");
  if (L.hk0 < 0 || L.hk1 > HkvT || L.hk0 >= L.hk1) return set_error(FP4ATTN_ERR_ARG, "bad KV-head range");
  if (Tp % 128 != 0 || Tp < T) return set_error(FP4ATTN_ERR_ARG, "Tp must be a multiple of 128 >= T");
  if (!L.q_codes || !L.q_scales || !L.q_g || !L.k_codes || !L.k_scales || !L.k_g || !L.v_hi || !L.v_lo || !L.out)
    return set_error(FP4ATTN_ERR_ARG, "null pointer");
  const bool dq = L.q_codes_lo != nullptr;
  if (L.flags & ~(FP4ATTN_DUAL_P | FP4ATTN_OUT_BF16 | FP4ATTN_PV_FP16)) return set_error(FP4ATTN_ERR_ARG, "bad flags");
  const bool dual_p = (L.flags & FP4ATTN_DUAL_P) != 0;
  if (dq && (!L.q_scales_lo || !L.q_g_lo)) return set_error(FP4ATTN_ERR_ARG, "null pointer (residual Q slice)");
  if (((uintptr_t)L.q_codes | (uintptr_t)L.k_codes | (uintptr_t)L.v_hi | (uintptr_t)L.v_lo | (uintptr_t)L.q_scales |
       (uintptr_t)L.k_scales | (uintptr_t)L.q_g | (uintptr_t)L.k_g | (uintptr_t)L.out | (uintptr_t)L.q_codes_lo |
       (uintptr_t)L.q_scales_lo | (uintptr_t)L.q_g_lo | (uintptr_t)L.row_max) % 16)
    return set_error(FP4ATTN_ERR_ARG, "buffers must be 16-byte aligned");
  const int G = HqT / HkvT;
  CUtensorMap mq, mql, mk, mvh, mvl;
  if (int e = encode_tiled_2d(&mq, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.q_codes, (uint64_t)HqT * (HD / 2),
                              (uint64_t)B * Tp, (uint64_t)HqT * (HD / 2), HD / 2, 128, CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  if (dq) {
    if (int e = encode_tiled_2d(&mql, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.q_codes_lo, (uint64_t)HqT * (HD / 2),
                                (uint64_t)B * Tp, (uint64_t)HqT * (HD / 2), HD / 2, 128, CU_TENSOR_MAP_SWIZZLE_64B))
      return e;
  } else {
    mql = mq;  // not read
  }
  if (int e = encode_tiled_2d(&mk, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.k_codes, (uint64_t)HkvT * (HD / 2),
                              (uint64_t)B * Tp, (uint64_t)HkvT * (HD / 2), HD / 2, 128, CU_TENSOR_MAP_SWIZZLE_64B))
    return e;
  if (int e = encode_tiled_2d(&mvh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, L.v_hi, (uint64_t)Tp, (uint64_t)B * HkvT * HD,
                              (uint64_t)Tp * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  if (int e = encode_tiled_2d(&mvl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, L.v_lo, (uint64_t)Tp, (uint64_t)B * HkvT * HD,
                              (uint64_t)Tp * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  AttnArgs a{};
  a.qsf = L.q_scales;
  a.gq = L.q_g;
  a.qsf_lo = L.q_scales_lo;
  a.gq_lo = L.q_g_lo;
  a.ksf = L.k_scales;
  a.gk = L.k_g;
  a.out = L.out;
  a.out_bf16 = (L.flags & FP4ATTN_OUT_BF16) ? 1 : 0;
  a.B = B;
  a.Hkv = L.hk1 - L.hk0;
  a.Hq = a.Hkv * G;
  a.T = T;
  a.Tp = Tp;
  a.hq0 = L.hk0 * G;
  a.hk0 = L.hk0;
  a.nkb4q = 2 * HqT;
  a.nkb4k = 2 * HkvT;
  a.HkvT = HkvT;
  a.HqT = HqT;
  a.pv_lo_tiles = (L.flags & FP4ATTN_PV_FP16) ? 1 : 0x7FFFFFFF;
  // precomputed row maxima: single-slice Q with a scratch for them (the traced kernel keeps its max pass)
  const bool pre = L.row_max != nullptr && !dq;
  a.row_max = pre ? L.row_max : nullptr;
  a.causal = L.causal ? 1 : 0;
  a.scale_log2 = L.scaling * 1.4426950408889634f;
  a.units = B * a.Hq * (Tp / 128);
  // the event timeline is recorded by the one-group single-slice kernel only
  a.trace = (dq || dual_p) ? nullptr : g_trace;
  using Kern = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
                        AttnArgs);
  static const Kern kerns[8] = {fp4_attn_kernel<false, false, false, false>, fp4_attn_kernel<false, true, false, false>,
                                fp4_attn_kernel<false, false, true, false>,  fp4_attn_kernel<false, true, true, false>,
                                fp4_attn_kernel<false, false, false, true>,  fp4_attn_kernel<false, false, true, true>,
                                fp4_attn_kernel<true, false, false, false>,  fp4_attn_kernel<true, false, false, true>};
  const Kern kern = a.trace ? kerns[6 + (pre ? 1 : 0)]
                    : pre   ? kerns[4 + (dual_p ? 1 : 0)]
                            : kerns[(dq ? 1 : 0) + (dual_p ? 2 : 0)];
  if (int e = set_smem_attr((const void*)kern, SMEM_BYTES)) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int grid = L.num_ctas > 0 ? L.num_ctas : sms;
  if (grid > a.units) grid = a.units;
  if (pre) {
    // K codes two key tiles per box, and a 32-bit view of the K scale atoms ([B*Tp/128] row blocks of
    // HkvT * 1024 bytes) boxed two row blocks at a time
    CUtensorMap mk2, mksf;
    if (int e = encode_tiled_2d(&mk2, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.k_codes, (uint64_t)HkvT * (HD / 2),
                                (uint64_t)B * Tp, (uint64_t)HkvT * (HD / 2), HD / 2, 256, CU_TENSOR_MAP_SWIZZLE_64B))
      return e;
    if (int e = encode_tiled_2d(&mksf, CU_TENSOR_MAP_DATA_TYPE_UINT32, L.k_scales, (uint64_t)HkvT * 256,
                                (uint64_t)B * Tp / 128, (uint64_t)HkvT * 1024, 256, 2, CU_TENSOR_MAP_SWIZZLE_NONE))
      return e;
    if (int e = set_smem_attr((const void*)fp4_rowmax_t_kernel, rmt::SMEM_BYTES)) return e;
    fp4_rowmax_t_kernel<<<grid, rmt::THREADS, rmt::SMEM_BYTES, st>>>(mq, mk2, mksf, a);
    if (int e = check_launch("fp4_rowmax_t_kernel")) return e;
    if (!dual_p && !a.trace && pingpong_enabled()) {
      if (int e = set_smem_attr((const void*)fp4_attn_pingpong_kernel, pp::SMEM_BYTES)) return e;
      fp4_attn_pingpong_kernel<<<grid, pp::THREADS, pp::SMEM_BYTES, st>>>(mq, mk, mvh, mvl, a);
      return check_launch("fp4_attn_pingpong_kernel");
    }
  }
  kern<<<grid, THREADS, SMEM_BYTES, st>>>(mq, mql, mk, mvh, mvl, a);
  return check_launch("fp4_attn_kernel");
}

extern "C" int fp4attn_fwd_packed_dual(const uint8_t* q_codes, const uint8_t* q_scales, const float* q_g,
                                       const uint8_t* q_codes_lo, const uint8_t* q_scales_lo, const float* q_g_lo,
                                       const uint8_t* k_codes, const uint8_t* k_scales, const float* k_g,
                                       const uint16_t* v_hi, const uint16_t* v_lo, void* out, int B, int Hq,
                                       int Hkv, int T, int Tp, int D, int causal, float scaling, int flags,
                                       int num_ctas, void* stream) {
  clear_error();
  AttnLaunch L{q_codes, q_scales, q_g, q_codes_lo, q_scales_lo, q_g_lo, k_codes, k_scales, k_g, v_hi, v_lo,
               out,     nullptr,  B,   Hq,         Hkv,         T,      Tp,      D,        0,   Hkv,  causal,
               scaling, flags,    num_ctas};
  return launch_attention(L, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int fp4attn_fwd_packed_heads(const uint8_t* q_codes, const uint8_t* q_scales, const float* q_g,
                                        const uint8_t* q_codes_lo, const uint8_t* q_scales_lo, const float* q_g_lo,
                                        const uint8_t* k_codes, const uint8_t* k_scales, const float* k_g,
                                        const uint16_t* v_hi, const uint16_t* v_lo, float* row_max, void* out,
                                        int B, int Hq, int Hkv, int T, int Tp, int D, int hkv0, int hkv1, int causal,
                                        float scaling, int flags, void* stream) {
  clear_error();
  AttnLaunch L{q_codes, q_scales, q_g, q_codes_lo, q_scales_lo, q_g_lo, k_codes, k_scales, k_g,  v_hi, v_lo,
               out,     row_max,  B,   Hq,         Hkv,         T,      Tp,      D,        hkv0, hkv1, causal,
               scaling, flags,    0};
  return launch_attention(L, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int fp4attn_fwd_packed(const uint8_t* q_codes, const uint8_t* q_scales, const float* q_g,
                                  const uint8_t* k_codes, const uint8_t* k_scales, const float* k_g,
                                  const uint16_t* v_hi, const uint16_t* v_lo, float* out, int B, int Hq, int Hkv,
                                  int T, int Tp, int D, int causal, float scaling, int num_ctas, void* stream) {
  return fp4attn_fwd_packed_dual(q_codes, q_scales, q_g, nullptr, nullptr, nullptr, k_codes, k_scales, k_g, v_hi, v_lo,
                                 out, B, Hq, Hkv, T, Tp, D, causal, scaling, 0, num_ctas, stream);
}
