// attn_pingpong.cuh -- single-pass NVFP4 attention with two groups of softmax
// warps that take alternate key tiles (included by attention.cu, which defines
// AttnArgs, the unit order and the softmax arithmetic it uses).
//
// Same computation as fp4_attn_kernel with precomputed row maxima
// (llama_patch.py:57-105 on the NVFP4 operands of llama_patch.py:167-196):
// e = exp2(z*u - m*u) with the exact row maximum m from fp4_rowmax_t_kernel, the
// row sum l = sum e, P-hat = NVFP4 fake-quant of e per 16 keys (E4M3 block
// scale, E2M1 round-to-nearest-even), O = (P-hat V-hat) / l.  The chunk
// arithmetic is chunk_p, so a key tile's P-hat is bit for bit the one
// fp4_attn_kernel forms.
//
// Schedule.  With one group of sixteen softmax warps on every tile, the SM
// idles while all of them wait for the same S buffer or hand the same P-hat
// to the PV thread.  Here tile t (counted over the CTA's units) belongs to
// group t & 1: eight warps, warp (quarter, half) owning rows 32*quarter ..
// +31 and key columns 64*half .. +63 of its group's tiles.  Each group has
// its own S buffer in TMEM, so one group computes while the other loads its
// scores or stores its P-hat, and the tensor pipe sees QK and PV of both.
// P-hat has one TMEM buffer: a group stores tile t's P-hat once PV(t-1) has
// read the previous one, so PV runs strictly in tile order.  (Handing P-hat
// over in two halves of 64 keys, so that the next tile's first half is stored
// while PV still runs on the second, measured slower: the extra wait costs the
// PV thread more than the overlap gains.)  The tensor pipe is what bounds the kernel
// (8 kind::f16 MMAs of ~100 cycles per tile for PV, 2 mxf4nvf4 MMAs and 2
// scale-atom copies for QK), so each tile carries only the commits it needs:
// the PV thread releases the K stage (the group is done with its gk when it
// hands over P-hat), and P-hat's release also frees the V-hat stage.
//
// TMEM: S0 [0,128), S1 [128,256), O [256,384), P-hat [384,448) (fp16; keys
// 32c .. 32c+31 at columns 16c .. 16c+15), Q scale atoms per Q stage from
// 448, K scale atoms per K stage from 464.
//
// A unit's output is written by both groups (group g: O columns 64g .. +63)
// once its last PV has finished; the row sum comes from four partials (two
// groups x two column halves) in a 4-slot shared-memory ring.  A group runs
// the epilogues of finished units just before it next stores a P-hat (or
// before it reuses a partial slot, or at the end), so its warps are not idle
// while a unit's last PV drains.  Every wait is bounded (mbar_wait): on a
// timeout the kernel records the site and runs to its end.
#pragma once

namespace pp {
constexpr int BM = 128, BN = 128, HD = 128;
constexpr int NQ = 2;   // Q stages (the next unit's Q lands while this one runs)
constexpr int NK = 4;   // K stages
constexpr int NV = 2;   // V-hat stages (hi and lo planes of 128 keys)
constexpr int GW = 8;   // warps per softmax group
constexpr int THREADS = 128 + 2 * GW * 32;
constexpr int NL = 4;   // row-sum partial slots (units in flight between the two groups)
// shared memory (bytes from a 1024-aligned base)
constexpr int Q_STAGE = 10240;  // codes 8 KB, scale atoms 1 KB (+8192), g 512 B (+9216), row maxima 512 B (+9728)
constexpr int OFF_Q = 0;
constexpr int K_STAGE = 10240;  // codes 8 KB, scale atoms 1 KB (+8192), gk 512 B (+9216)
constexpr int OFF_K = OFF_Q + NQ * Q_STAGE;
constexpr int V_HALF = HD * 64 * 2;  // 128 channels x 64 keys x fp16 (one TMA box)
constexpr int V_STAGE = 4 * V_HALF;  // keys 0-63 hi, lo; keys 64-127 hi, lo
constexpr int OFF_V = OFF_K + NK * K_STAGE;
constexpr int OFF_L = OFF_V + NV * V_STAGE;         // [NL][4 partials][128 rows] fp32
constexpr int OFF_BAR = OFF_L + NL * 4 * 128 * 4;
constexpr int SMEM_BYTES = OFF_BAR + 512 + 1024;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t T_S = 0, T_O = 256, T_P = 384, T_SFA = 448, T_SFB = T_SFA + 8 * NQ;
static_assert(OFF_V % 1024 == 0, "V-hat stages need 1024-byte alignment (128-byte swizzle)");
static_assert(T_SFB + 8 * NK <= TMEM_COLS, "TMEM columns");
static_assert(SMEM_BYTES <= 232448, "shared memory map exceeds the 227 KB a CTA can have");
}  // namespace pp

__global__ void __launch_bounds__(pp::THREADS, 1)
    fp4_attn_pingpong_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                             const __grid_constant__ CUtensorMap tmVhi, const __grid_constant__ CUtensorMap tmVlo,
                             AttnArgs p) {
  using namespace pp;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* lpart = reinterpret_cast<float*>(sm + OFF_L);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* q_full = bar;              // [NQ]
  uint64_t* q_empty = q_full + NQ;     // [NQ] MMA commit + every softmax warp (they read g and m)
  uint64_t* k_full = q_empty + NQ;     // [NK]
  uint64_t* k_empty = k_full + NK;     // [NK] the PV thread, for the softmax warps (their last gk read)
  uint64_t* v_full = k_empty + NK;     // [NV]
  uint64_t* s_full = v_full + NV;      // [2] per group: its S buffer written
  uint64_t* s_free = s_full + 2;       // [2] per group: every warp of the group has loaded it
  uint64_t* p_full = s_free + 2;       // [2] per tile parity: the group stored its P-hat
  uint64_t* p_free = p_full + 2;       // [2] per tile parity: PV has read that P-hat (and its V-hat stage)
  uint64_t* o_full = p_free + 2;       // a unit's last PV finished
  uint64_t* o_free = o_full + 1;       // every softmax warp has read O
  uint64_t* l_full = o_free + 1;       // [NL] every softmax warp wrote its row-sum partial
  uint64_t* l_free = l_full + NL;      // [NL] every softmax warp read the slot
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(l_free + NL);
  static_assert(2 * NQ + 2 * NK + NV + 10 + 2 * NL + 1 <= 64, "barriers exceed their 512-byte slot");
  static_assert(NV == 2, "a V-hat stage is released with the P-hat of the same tile parity");

  const int warp = threadIdx.x / 32;
  const int group = p.Hq / p.Hkv;  // query heads per KV head
  if (threadIdx.x == 0) {
    for (int i = 0; i < NQ; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1 + 2 * GW);
    }
    for (int i = 0; i < NK; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < NV; ++i) mbar_init(&v_full[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], GW);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], GW);
      mbar_init(&p_free[i], 1);
    }
    mbar_init(o_full, 1);
    mbar_init(o_free, 2 * GW);
    for (int i = 0; i < NL; ++i) {
      mbar_init(&l_full[i], 2 * GW);
      mbar_init(&l_free[i], 2 * GW);
    }
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

  if (warp == 0) {
    // ------------------------------------------------- producer: Q and K
    if (elect_one_lane()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      uint32_t kc = 0, uc = 0;
      for (int i = 0, u = cta_unit(0, p.units); u >= 0; u = cta_unit(++i, p.units), ++uc) {
        const Unit un = unit_of(u, p);
        const int n = kv_tiles(un, p);
        const int hq = p.hq0 + un.h, hk = p.hk0 + un.h / group;
        const int qrow = un.b * p.Tp + un.qt * BM;
        const int qs = uc & 1;
        uint8_t* qb = sm + OFF_Q + qs * Q_STAGE;
        if (uc >= NQ) mbar_wait(&q_empty[qs], ((uc >> 1) - 1) & 1, 0x601);
        mbar_arrive_expect_tx(&q_full[qs], 8192 + 1024 + 512 + 512);
        tma_load_2d(qb, &tmQ, &q_full[qs], hq * (HD / 2), qrow);
        bulk_load(qb + 8192, p.qsf + ((int64_t)(qrow / 128) * p.nkb4q + 2 * hq) * 512, 1024, &q_full[qs]);
        bulk_load(qb + 9216, p.gq + qrow, 512, &q_full[qs]);
        bulk_load(qb + 9728, p.row_max + ((int64_t)un.b * p.HqT + hq) * p.Tp + un.qt * BM, 512, &q_full[qs]);
        for (int j = 0; j < n; ++j, ++kc) {
          const int s = kc % NK;
          if (kc >= NK) mbar_wait(&k_empty[s], ((kc / NK) - 1) & 1, 0x602);
          uint8_t* ks = sm + OFF_K + s * K_STAGE;
          const int krow = un.b * p.Tp + j * BN;
          mbar_arrive_expect_tx(&k_full[s], 8192 + 1024 + 512);
          tma_load_2d(ks, &tmK, &k_full[s], hk * (HD / 2), krow);
          bulk_load(ks + 8192, p.ksf + ((int64_t)(krow / 128) * p.nkb4k + 2 * hk) * 512, 1024, &k_full[s]);
          bulk_load(ks + 9216, p.gk + krow, 512, &k_full[s]);
        }
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------- producer: V-hat tiles
    if (elect_one_lane()) {
      tma_prefetch_desc(&tmVhi);
      tma_prefetch_desc(&tmVlo);
      uint32_t vc = 0;
      for (int i = 0, u = cta_unit(0, p.units); u >= 0; u = cta_unit(++i, p.units)) {
        const Unit un = unit_of(u, p);
        const int n = kv_tiles(un, p);
        const int vrow = (un.b * p.HkvT + p.hk0 + un.h / group) * HD;
        const bool lo = un.qt < p.pv_lo_tiles;  // the lo plane only where PV reads it
        for (int j = 0; j < n; ++j, ++vc) {
          const int vs = vc % NV;
          if (vc >= NV) mbar_wait(&p_free[vs], ((vc / NV) - 1) & 1, 0x603);
          uint8_t* v = sm + OFF_V + vs * V_STAGE;
          mbar_arrive_expect_tx(&v_full[vs], lo ? V_STAGE : V_STAGE / 2);
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            tma_load_2d(v + 2 * half * V_HALF, &tmVhi, &v_full[vs], j * BN + 64 * half, vrow);
            if (lo) tma_load_2d(v + (2 * half + 1) * V_HALF, &tmVlo, &v_full[vs], j * BN + 64 * half, vrow);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- QK^T issue
    // S(t) goes to the S buffer of group t & 1 once that group has loaded S(t - 2).
    if (elect_one_lane()) {
      const uint32_t idq = idesc_nvf4(BM, BN);
      uint32_t t = 0, uc = 0;
      for (int i = 0, u = cta_unit(0, p.units); u >= 0; u = cta_unit(++i, p.units), ++uc) {
        const Unit un = unit_of(u, p);
        const int n = kv_tiles(un, p);
        const int qs = uc & 1;
        const uint8_t* qb = sm + OFF_Q + qs * Q_STAGE;
        const uint32_t sfa = tmem + T_SFA + 8 * qs;
        mbar_wait(&q_full[qs], (uc >> 1) & 1, 0x611);
        tc_fence_after();
        tmem_cp_sf_atom(sfa, smem_desc(smem_u32(qb + 8192), 16, 128, kSwizzleNone));
        tmem_cp_sf_atom(sfa + 4, smem_desc(smem_u32(qb + 8192 + 512), 16, 128, kSwizzleNone));
        for (int j = 0; j < n; ++j, ++t) {
          const int g = t & 1, s = t % NK;
          if (t >= 2) mbar_wait(&s_free[g], ((t >> 1) - 1) & 1, 0x612);
          mbar_wait(&k_full[s], (t / NK) & 1, 0x613);
          tc_fence_after();
          uint8_t* ks = sm + OFF_K + s * K_STAGE;
          const uint32_t sfb = tmem + T_SFB + 8 * s;
          tmem_cp_sf_atom(sfb, smem_desc(smem_u32(ks + 8192), 16, 128, kSwizzleNone));
          tmem_cp_sf_atom(sfb + 4, smem_desc(smem_u32(ks + 8192 + 512), 16, 128, kSwizzleNone));
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const uint64_t ad = smem_desc(smem_u32(qb) + kk * 32, 16, 512, kSwizzle64B);
            const uint64_t bd = smem_desc(smem_u32(ks) + kk * 32, 16, 512, kSwizzle64B);
            mma_nvf4(tmem + T_S + 128 * g, ad, bd, idq, sfa + 4 * kk, sfb + 4 * kk, kk > 0 ? 1u : 0u);
          }
          tc_commit(&s_full[g]);
        }
        tc_commit(&q_empty[qs]);
      }
    }
  } else if (warp == 3) {
    // --------------------------------------------------------- PV issue
    // O += P-hat(t) V-hat(t) in tile order, once the tile's group has stored P-hat(t);
    // the commit frees the P-hat buffer for tile t + 1 (the other group).
    if (elect_one_lane()) {
      const uint32_t idv = idesc_f16(BM, HD);
      uint32_t t = 0, uc = 0;
      for (int i = 0, u = cta_unit(0, p.units); u >= 0; u = cta_unit(++i, p.units), ++uc) {
        const Unit un = unit_of(u, p);
        const int n = kv_tiles(un, p);
        const int parts = un.qt < p.pv_lo_tiles ? 2 : 1;  // hi + lo planes, or hi alone
        for (int j = 0; j < n; ++j, ++t) {
          const int par = t & 1, vs = t % NV;
          mbar_wait(&v_full[vs], (t / NV) & 1, 0x621);
          mbar_wait(&p_full[par], (t >> 1) & 1, 0x622);
          mbar_arrive(&k_empty[t % NK]);  // P-hat stored: the group is done with the stage's gk
          if (j == 0 && uc > 0) mbar_wait(o_free, (uc - 1) & 1, 0x623);
          tc_fence_after();
          const uint32_t v = smem_u32(sm + OFF_V + vs * V_STAGE);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {  // keys 16kk .. 16kk+15
            const uint32_t a = tmem + T_P + 8 * kk;
            for (int part = 0; part < parts; ++part) {
              const uint32_t vb = v + ((kk >> 2) * 2 + part) * V_HALF + (kk & 3) * 32;
              mma_f16_ts(tmem + T_O, a, smem_desc(vb, 16, 1024, kSwizzle128B), idv,
                         (j > 0 || kk > 0 || part > 0) ? 1u : 0u);
            }
          }
          tc_commit(&p_free[par]);
        }
        tc_commit(o_full);
      }
    }
  } else {
    // ------------------------------------------------- softmax groups
    const int sw = warp - 4;
    const int grp = sw / GW;          // tiles t with t & 1 == grp
    const int half = (sw / 4) & 1;    // key columns 64*half .. +63 of each tile
    const int quarter = warp & 3;     // TMEM lane quarter this warp may access
    const int r = quarter * 32 + (threadIdx.x & 31);  // row of the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const bool wlead = (threadIdx.x & 31) == 0;
    const float r6 = __frcp_rn(6.0f);
    const int c0 = 64 * half;  // first of this warp's two 32-key chunks
    const uint32_t s_cols = tmem + lane_base + T_S + 128 * grp;
    const int part_idx = grp * 2 + half;  // this warp's row-sum partial
    uint32_t pend_lo = 0, pend_hi = 0;    // units [pend_lo, pend_hi) whose O this warp still writes

    // O of CTA unit i / l: this warp's 32 columns (64*grp + 32*half) of its row; then O and
    // the partial slot are released.
    auto epilogue = [&](uint32_t i) {
      mbar_wait(o_full, i & 1, 0x631);
      mbar_wait(&l_full[i % NL], (i / NL) & 1, 0x632);
      tc_fence_after();
      const float* lp = lpart + (i % NL) * 512;
      const float l = (lp[r] + lp[128 + r]) + (lp[256 + r] + lp[384 + r]);
      const float rl = 1.0f / l;
      const int col = 64 * grp + 32 * half;
      uint32_t a[32];
      tmem_ld32(tmem + lane_base + T_O + col, a);
      tmem_ld_wait();
      const Unit un = unit_of(cta_unit((int)i, p.units), p);
      const int qpos = un.qt * BM + r;
      if (qpos < p.T) {
        const int64_t off = (((int64_t)un.b * p.T + qpos) * p.Hq + un.h) * HD + col;
        if (p.out_bf16) {  // rounded to bf16 as the reference's bf16 matmul output is
          uint4* d4 = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + off);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __nv_bfloat162 h2 = __floats2bfloat162_rn(__uint_as_float(a[8 * k + 2 * e]) * rl,
                                                              __uint_as_float(a[8 * k + 2 * e + 1]) * rl);
              w[e] = *reinterpret_cast<const uint32_t*>(&h2);
            }
            d4[k] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        } else {
          float4* d4 = reinterpret_cast<float4*>(static_cast<float*>(p.out) + off);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            d4[k] = make_float4(__uint_as_float(a[4 * k]) * rl, __uint_as_float(a[4 * k + 1]) * rl,
                                __uint_as_float(a[4 * k + 2]) * rl, __uint_as_float(a[4 * k + 3]) * rl);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (wlead) {
        mbar_arrive(o_free);
        mbar_arrive(&l_free[i % NL]);
      }
    };

    uint32_t t = 0, uc = 0;
    for (int i = 0, u = cta_unit(0, p.units); u >= 0; u = cta_unit(++i, p.units), ++uc) {
      const Unit un = unit_of(u, p);
      const int n = kv_tiles(un, p);
      const int qs = uc & 1;
      const uint8_t* qb = sm + OFF_Q + qs * Q_STAGE;
      mbar_wait(&q_full[qs], (uc >> 1) & 1, 0x633);
      const float uscale = reinterpret_cast<const float*>(qb + 9216)[r] * p.scale_log2;
      const float m = reinterpret_cast<const float*>(qb + 9728)[r];
      __syncwarp();
      if (wlead) mbar_arrive(&q_empty[qs]);  // g and m are in registers
      const float mu = m == -INFINITY ? 0.0f : m * uscale;
      const uint64_t u2 = pk2(uscale, uscale), nmu2 = pk2(-mu, -mu);
      uint64_t lsum2[4] = {pk2(0.0f, 0.0f), pk2(0.0f, 0.0f), pk2(0.0f, 0.0f), pk2(0.0f, 0.0f)};
      // this group's first tile of the unit: t + ((t & 1) != grp)
      for (int j = (int)((t & 1) != (uint32_t)grp); j < n; j += 2) {
        const uint32_t tt = t + j;  // tt & 1 == grp
        mbar_wait(&s_full[grp], (tt >> 1) & 1, 0x634);
        tc_fence_after();
        const uint32_t gk = smem_u32(sm + OFF_K + (tt % NK) * K_STAGE + 9216) + 4 * c0;
        // keys with column > lim are masked (causal diagonal tile, or keys past T)
        const int lim = (p.causal && j == un.qt) ? r : (p.T - 1 - j * BN);
        uint32_t a[32], pk0[16], pk1[16];
        tmem_ld32(s_cols + c0, a);
        tmem_ld_wait();
        if (lim < c0 + 31) chunk_p<true>(a, gk, c0, lim, u2, nmu2, r6, lsum2, pk0);
        else chunk_p<false>(a, gk, c0, lim, u2, nmu2, r6, lsum2, pk0);
        tmem_ld32(s_cols + c0 + 32, a);
        tmem_ld_wait();
        // both chunks are in registers: the group's S buffer may take S(tt + 2)
        tc_fence_before();
        __syncwarp();
        if (wlead) mbar_arrive(&s_free[grp]);
        if (lim < c0 + 63) chunk_p<true>(a, gk + 128, c0 + 32, lim, u2, nmu2, r6, lsum2, pk1);
        else chunk_p<false>(a, gk + 128, c0 + 32, lim, u2, nmu2, r6, lsum2, pk1);
        // outputs of finished units first (their last PV precedes PV(tt - 1))
        while (pend_lo < pend_hi) epilogue(pend_lo++);
        // the P-hat buffer is free once PV(tt - 1) has read it
        if (tt >= 1) mbar_wait(&p_free[(tt - 1) & 1], ((tt - 1) >> 1) & 1, 0x635);
        tc_fence_after();
        tmem_st16(tmem + lane_base + T_P + 32 * half, pk0);
        tmem_st16(tmem + lane_base + T_P + 32 * half + 16, pk1);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (wlead) mbar_arrive(&p_full[grp]);
      }
      t += n;
      // the unit's row-sum partial of this warp (zero when the group had no tile in it)
      float l0, l1;
      upk2(add2(add2(lsum2[0], lsum2[1]), add2(lsum2[2], lsum2[3])), l0, l1);
      if (uc >= NL) {
        // the slot's previous unit must be read by every warp, this one included
        while (pend_lo + NL <= uc) epilogue(pend_lo++);
        mbar_wait(&l_free[uc % NL], ((uc / NL) - 1) & 1, 0x636);
      }
      lpart[(uc % NL) * 512 + part_idx * 128 + r] = l0 + l1;
      __syncwarp();
      if (wlead) mbar_arrive(&l_full[uc % NL]);
      pend_hi = uc + 1;
    }
    while (pend_lo < pend_hi) epilogue(pend_lo++);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}
