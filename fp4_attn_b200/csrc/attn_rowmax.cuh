// attn_rowmax.cuh -- row maxima of the scores for the single-pass attention
// kernels, with three groups of max warps that each own whole work units
// (included by attention.cu, which defines AttnArgs, the unit order and
// chunk_max).
//
// fp4_rowmax_groups_kernel writes, for every query row of every unit, the
// exact maximum over its keys of z = (Q-hat K-hat^T) * gk: the same tcgen05
// kind::mxf4nvf4 products (M=128, N=128, K=64) of the same operands, reduced
// by the same chunk_max, so the maxima equal the ones the two-pass attention
// kernel finds in its first pass (the reference's P / rowmax(P) needs them
// before any P is quantized, llama_patch.py:76-99).
//
// Schedule.  The max of a 128 x 128 tile is a few dozen instructions per
// warp and its MMAs take ~134 cycles of the tensor pipe, but one thread
// issuing a tile (two waits, two scale-atom copies, two MMAs, a commit and
// its loop) needs ~1000 cycles.  So three groups each own every third unit
// of the CTA, one S buffer and one issuing thread (warp 1 + g): while one
// thread waits, the others issue.  A group's four max warps (one per TMEM
// lane quarter) reduce all 128 columns of their 32 rows and release the S
// buffer and the K stage (the MMA has read the stage once its scores are
// visible).  The producer loads the groups' tiles round robin (one tile per
// group per round, exhausted groups skipped) into the K ring; a group finds
// the stage of its r-th tile from the three groups' tile counts.  TMEM: S
// buffers [0,384), Q scale atoms per (group, Q stage) from 384, K scale atoms
// per group from 432.  Every wait is bounded.
#pragma once

namespace rmg {
constexpr int NG = 3;   // groups, one S buffer each
constexpr int NK = 8;   // K stages
constexpr int THREADS = 128 + NG * 128;
constexpr int Q_STAGE = 9216;  // codes 8 KB, scale atoms 1 KB (+8192); two stages per group
constexpr int OFF_Q = 0;
constexpr int K_STAGE = 10240;  // codes 8 KB, scale atoms 1 KB (+8192), gk 512 B (+9216)
constexpr int OFF_K = OFF_Q + NG * 2 * Q_STAGE;
constexpr int OFF_BAR = OFF_K + NK * K_STAGE;
constexpr int SMEM_BYTES = OFF_BAR + 512 + 1024;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t T_SFA = NG * 128, T_SFB = T_SFA + 8 * 2 * NG;
static_assert(OFF_K % 1024 == 0 && Q_STAGE % 1024 == 0, "TMA destinations need 1024-byte alignment");
static_assert(T_SFB + 8 * NG <= TMEM_COLS, "TMEM columns");
static_assert(SMEM_BYTES <= 232448, "shared memory map");
}  // namespace rmg

// One group's walk over its units (CTA units g, g + NG, ...): the current unit,
// its tile count, the current tile and how many units the group has started.
struct RmgStream {
  int i, u, n, j;
  uint32_t k;
  Unit un;
  __device__ __forceinline__ void start(int g, const AttnArgs& p) {
    i = g;
    u = cta_unit(i, p.units);
    j = 0;
    k = 0;
    if (u >= 0) {
      un = unit_of(u, p);
      n = kv_tiles(un, p);
    }
  }
  __device__ __forceinline__ void next(const AttnArgs& p) {
    if (++j < n) return;
    j = 0;
    ++k;
    i += rmg::NG;
    u = cta_unit(i, p.units);
    if (u >= 0) {
      un = unit_of(u, p);
      n = kv_tiles(un, p);
    }
  }
};

// Tiles of all of group g's units.
__device__ __forceinline__ int rmg_tiles(int g, const AttnArgs& p) {
  int t = 0;
  for (int i = g, u = cta_unit(i, p.units); u >= 0; i += rmg::NG, u = cta_unit(i, p.units))
    t += kv_tiles(unit_of(u, p), p);
  return t;
}

__global__ void __launch_bounds__(rmg::THREADS, 1)
    fp4_rowmax_groups_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                             AttnArgs p) {
  using namespace rmg;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* q_full = bar;                // [NG][2]
  uint64_t* q_empty = q_full + 2 * NG;   // [NG][2] MMA commit after the unit's last QK
  uint64_t* k_full = q_empty + 2 * NG;   // [NK]
  uint64_t* k_empty = k_full + NK;       // [NK] the tile's four max warps (after its scores, they read gk)
  uint64_t* s_full = k_empty + NK;       // [NG]
  uint64_t* s_free = s_full + NG;        // [NG] the group's four warps have loaded the buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_free + NG);
  static_assert(4 * NG + 2 * NK + 2 * NG + 1 <= 64, "barriers exceed their 512-byte slot");
  const int warp = threadIdx.x / 32;
  const int group = p.Hq / p.Hkv;  // query heads per KV head
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2 * NG; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < NK; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 4);
    }
    for (int i = 0; i < NG; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
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
    // ------------------------------------------------- producer: Q and K, round robin over the groups
    if (elect_one_lane()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      RmgStream st[NG];
#pragma unroll
      for (int g = 0; g < NG; ++g) st[g].start(g, p);
      uint32_t seq = 0;
      for (bool any = true; any;) {
        any = false;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          RmgStream& s = st[g];
          if (s.u < 0) continue;
          any = true;
          if (s.j == 0) {
            const int qs = 2 * g + (int)(s.k & 1);
            uint8_t* qb = sm + OFF_Q + qs * Q_STAGE;
            const int hq = p.hq0 + s.un.h;
            const int qrow = s.un.b * p.Tp + s.un.qt * attn::BM;
            if (s.k >= 2) mbar_wait(&q_empty[qs], ((s.k >> 1) - 1) & 1, 0x701);
            mbar_arrive_expect_tx(&q_full[qs], attn::Q_BYTES + 1024);
            tma_load_2d(qb, &tmQ, &q_full[qs], hq * (attn::HD / 2), qrow);
            bulk_load(qb + 8192, p.qsf + ((int64_t)(qrow / 128) * p.nkb4q + 2 * hq) * 512, 1024, &q_full[qs]);
          }
          const int ks = (int)(seq % NK);
          uint8_t* kb = sm + OFF_K + ks * K_STAGE;
          const int hk = p.hk0 + s.un.h / group;
          const int krow = s.un.b * p.Tp + s.j * attn::BN;
          if (seq >= NK) mbar_wait(&k_empty[ks], ((seq / NK) - 1) & 1, 0x702);
          mbar_arrive_expect_tx(&k_full[ks], 8192 + 1024 + 512);
          tma_load_2d(kb, &tmK, &k_full[ks], hk * (attn::HD / 2), krow);
          bulk_load(kb + 8192, p.ksf + ((int64_t)(krow / 128) * p.nkb4k + 2 * hk) * 512, 1024, &k_full[ks]);
          bulk_load(kb + 9216, p.gk + krow, 512, &k_full[ks]);
          ++seq;
          s.next(p);
        }
      }
    }
  } else if (warp <= NG) {
    // ------------------------------------------------- MMA issue, one thread per group
    const int g = warp - 1;
    int len[NG];
#pragma unroll
    for (int x = 0; x < NG; ++x) len[x] = rmg_tiles(x, p);
    if (elect_one_lane()) {
      const uint32_t idq = idesc_nvf4(attn::BM, attn::BN);
      const uint32_t sfb = tmem + T_SFB + 8 * g, sbuf = tmem + 128 * g;
      RmgStream s;
      s.start(g, p);
      for (uint32_t rr = 0; s.u >= 0; ++rr) {
        uint32_t seq = 0;  // ring position of this group's rr-th tile (see the max warps)
#pragma unroll
        for (int x = 0; x < NG; ++x) seq += (uint32_t)min(len[x], (int)rr) + ((x < g && len[x] > (int)rr) ? 1u : 0u);
        const int qs = 2 * g + (int)(s.k & 1);
        const uint8_t* qb = sm + OFF_Q + qs * Q_STAGE;
        const uint32_t sfa = tmem + T_SFA + 8 * qs;
        const int ks = (int)(seq % NK);
        const uint8_t* kb = sm + OFF_K + ks * K_STAGE;
        if (s.j == 0) {
          mbar_wait(&q_full[qs], (s.k >> 1) & 1, 0x703);
          tc_fence_after();
          tmem_cp_sf_atom(sfa, smem_desc(smem_u32(qb + 8192), 16, 128, kSwizzleNone));
          tmem_cp_sf_atom(sfa + 4, smem_desc(smem_u32(qb + 8192 + 512), 16, 128, kSwizzleNone));
        }
        if (rr >= 1) mbar_wait(&s_free[g], (rr - 1) & 1, 0x704);
        mbar_wait(&k_full[ks], (seq / NK) & 1, 0x705);
        tc_fence_after();
        tmem_cp_sf_atom(sfb, smem_desc(smem_u32(kb + 8192), 16, 128, kSwizzleNone));
        tmem_cp_sf_atom(sfb + 4, smem_desc(smem_u32(kb + 8192 + 512), 16, 128, kSwizzleNone));
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const uint64_t ad = smem_desc(smem_u32(qb) + kk * 32, 16, 512, kSwizzle64B);
          const uint64_t bd = smem_desc(smem_u32(kb) + kk * 32, 16, 512, kSwizzle64B);
          mma_nvf4(sbuf, ad, bd, idq, sfa + 4 * kk, sfb + 4 * kk, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[g]);
        if (s.j == s.n - 1) tc_commit(&q_empty[qs]);
        s.next(p);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------- max warps
    const int g = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + (threadIdx.x & 31);
    const uint32_t scols = tmem + ((uint32_t)(quarter * 32) << 16) + 128 * g;
    const bool wlead = (threadIdx.x & 31) == 0;
    int len[NG];
#pragma unroll
    for (int x = 0; x < NG; ++x) len[x] = rmg_tiles(x, p);
    RmgStream s;
    s.start(g, p);
    float m = -INFINITY;
    for (uint32_t rr = 0; s.u >= 0; ++rr) {
      // ring stage of this group's rr-th tile: the tiles of the earlier rounds, then the groups before g
      uint32_t seq = 0;
#pragma unroll
      for (int x = 0; x < NG; ++x) seq += (uint32_t)min(len[x], (int)rr) + ((x < g && len[x] > (int)rr) ? 1u : 0u);
      const uint32_t gk = smem_u32(sm + OFF_K + (seq % NK) * K_STAGE + 9216);
      const int lim = (p.causal && s.j == s.un.qt) ? r : (p.T - 1 - s.j * attn::BN);
      mbar_wait(&s_full[g], rr & 1, 0x706);
      tc_fence_after();
      uint32_t a0[32], a1[32];
      tmem_ld32(scols, a0);
      tmem_ld32(scols + 32, a1);
      tmem_ld_wait();
      m = lim < 31 ? chunk_max<true>(a0, gk, 0, lim, m) : chunk_max<false>(a0, gk, 0, lim, m);
      m = lim < 63 ? chunk_max<true>(a1, gk + 128, 32, lim, m) : chunk_max<false>(a1, gk + 128, 32, lim, m);
      tmem_ld32(scols + 64, a0);
      tmem_ld32(scols + 96, a1);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (wlead) mbar_arrive(&s_free[g]);
      m = lim < 95 ? chunk_max<true>(a0, gk + 256, 64, lim, m) : chunk_max<false>(a0, gk + 256, 64, lim, m);
      m = lim < 127 ? chunk_max<true>(a1, gk + 384, 96, lim, m) : chunk_max<false>(a1, gk + 384, 96, lim, m);
      __syncwarp();
      if (wlead) mbar_arrive(&k_empty[seq % NK]);
      if (s.j == s.n - 1) {
        p.row_max[((int64_t)s.un.b * p.HqT + p.hq0 + s.un.h) * p.Tp + s.un.qt * attn::BM + r] = m;
        m = -INFINITY;
      }
      s.next(p);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}
