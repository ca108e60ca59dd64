// attn_rowmax.cuh -- row maxima of the scores for the single-pass attention
// kernels (included by attention.cu, which defines AttnArgs and the unit
// order).
//
// fp4_rowmax_t_kernel writes, for every query row of every unit, the exact
// maximum over its keys of z = (Q-hat K-hat^T) * gk: the same tcgen05
// kind::mxf4nvf4 block-16 products of the same operands (M=128, N=128, K=64
// per instruction), with K as the A operand, so S^T lands in TMEM (a TMEM lane
// is a key, a column a query).  The reference's P / rowmax(P) needs these
// maxima before any P is quantized (llama_patch.py:76-99).
//
// Why transposed.  While the tensor core streams FP4 MMAs it reads ~120
// bytes of shared memory per cycle, and a warp's own shared-memory loads then
// wait ~10x longer (measured: 1300 cycles for a 32-key reduction that takes
// 130 with the tensor core idle).  With a lane per query row every thread
// needs every key's global scale gk, i.e. shared-memory loads in the inner
// loop; with a lane per key a thread needs one gk per tile, which it loads
// from global memory (L2) before waiting for the tile.  Each thread keeps a
// running element-wise maximum over the unit's tiles for its key lane and 32
// query columns, and reduces across lanes once per unit (a 31-shuffle
// transpose-reduce, then the four lane quarters through shared memory).
//
// Schedule.  Every mbarrier operation and copy issue is slow while the MMAs
// hold shared memory (an arrive + TMA + bulk copy from one thread: ~220 cycles
// alone, ~600 here), so a K stage holds two consecutive key tiles of a unit,
// loaded by two TMAs (the codes as one 256-row box, both tiles' scale atoms as
// one box of a 32-bit view of the atom array).  One thread issuing a tile (two
// waits, two scale-atom copies, two MMAs, two commits) needs ~1000 cycles
// against ~134 of tensor work, so three threads (warps 1-3) issue: thread b
// takes tiles t = b mod 3 into S buffer b.  Sixteen max warps (lane quarter =
// keys, four blocks of 32 query columns) reduce every tile; a max warp loads
// the next tile's gk while it reduces this one.  TMEM: S buffers [0,384), Q
// scale atoms per (issuer, Q stage) from 384, K scale atoms per issuer from
// 432.  Every wait is bounded.
#pragma once

namespace rmt {
constexpr int NS = 3;   // S buffers, one issuing thread each
constexpr int NK = 4;   // K stages of two key tiles
constexpr int THREADS = 128 + 4 * 128;
constexpr int Q_STAGE = 9216;  // codes 8 KB, scale atoms 1 KB (+8192)
constexpr int OFF_Q = 0;
constexpr int K_STAGE = 18432;  // codes of two tiles 16 KB, their scale atoms 2 KB (+16384)
constexpr int OFF_K = OFF_Q + 2 * Q_STAGE;
constexpr int OFF_STAT = OFF_K + NK * K_STAGE;  // [2 units][4 lane quarters][128 queries] partial maxima
constexpr int OFF_BAR = OFF_STAT + 2 * 4 * 128 * 4;
constexpr int SMEM_BYTES = OFF_BAR + 512 + 1024;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t T_SFQ = NS * 128, T_SFK = T_SFQ + 8 * 2 * NS;
static_assert(OFF_K % 1024 == 0 && Q_STAGE % 1024 == 0 && K_STAGE % 1024 == 0, "TMA destinations");
static_assert(T_SFK + 8 * NS <= TMEM_COLS, "TMEM columns");
static_assert(SMEM_BYTES <= 232448, "shared memory map");
}  // namespace rmt

// After a butterfly over the warp, lane l holds the maximum over the 32 lanes
// of v[l] (v: this lane's 32 values, destroyed).
__device__ __forceinline__ float warp_transpose_max(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? v[i] : v[i + off];
      const float keep = upper ? v[i + off] : v[i];
      v[i] = fmaxf(keep, __shfl_xor_sync(0xFFFFFFFFu, send, off));
    }
  }
  return v[0];
}

__global__ void __launch_bounds__(rmt::THREADS, 1)
    fp4_rowmax_t_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK2,
                        const __grid_constant__ CUtensorMap tmKsf, AttnArgs p) {
  using namespace rmt;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* stat = reinterpret_cast<float*>(sm + OFF_STAT);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* q_full = bar;              // [2]
  uint64_t* q_empty = q_full + 2;      // [2] each issuer commits once per unit
  uint64_t* k_full = q_empty + 2;      // [NK]
  uint64_t* k_empty = k_full + NK;     // [NK] the commits of the stage's two tiles' issuers
  uint64_t* s_full = k_empty + NK;     // [NS]
  uint64_t* s_free = s_full + NS;      // [NS] every max warp has loaded the buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_free + NS);
  static_assert(4 + 2 * NK + 2 * NS + 1 <= 64, "barriers exceed their 512-byte slot");
  const int warp = threadIdx.x / 32;
  const int group = p.Hq / p.Hkv;  // query heads per KV head
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], NS);
    }
    for (int i = 0; i < NK; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 2);
    }
    for (int i = 0; i < NS; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 16);
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
    // ------------------------------------------------- producer: Q per unit, K per tile
    if (elect_one_lane()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK2);
      tma_prefetch_desc(&tmKsf);
      uint32_t pc = 0, uc = 0;
      for (int i = 0, u = cta_unit(0, p.units); u >= 0; u = cta_unit(++i, p.units), ++uc) {
        const Unit un = unit_of(u, p);
        const int n = kv_tiles(un, p);
        const int hq = p.hq0 + un.h, hk = p.hk0 + un.h / group;
        const int qrow = un.b * p.Tp + un.qt * attn::BM;
        const int qs = uc & 1;
        uint8_t* qb = sm + OFF_Q + qs * Q_STAGE;
        if (uc >= 2) mbar_wait(&q_empty[qs], ((uc >> 1) - 1) & 1, 0x701);
        mbar_arrive_expect_tx(&q_full[qs], attn::Q_BYTES + 1024);
        tma_load_2d(qb, &tmQ, &q_full[qs], hq * (attn::HD / 2), qrow);
        bulk_load(qb + 8192, p.qsf + ((int64_t)(qrow / 128) * p.nkb4q + 2 * hq) * 512, 1024, &q_full[qs]);
        for (int j = 0; j < n; j += 2, ++pc) {  // tiles j, j + 1 (the second may lie past the unit: unused)
          const int ks = (int)(pc % NK);
          uint8_t* kb = sm + OFF_K + ks * K_STAGE;
          const int krow = un.b * p.Tp + j * attn::BN;
          if (pc >= NK) mbar_wait(&k_empty[ks], ((pc / NK) - 1) & 1, 0x702);
          mbar_arrive_expect_tx(&k_full[ks], 16384 + 2048);
          tma_load_2d(kb, &tmK2, &k_full[ks], hk * (attn::HD / 2), krow);
          tma_load_2d(kb + 16384, &tmKsf, &k_full[ks], hk * 256, krow / 128);
        }
      }
    }
  } else if (warp <= NS) {
    // ------------------------------------------------- MMA issue: thread b takes tiles t = b mod NS
    const int b = warp - 1;
    if (elect_one_lane()) {
      const uint32_t idq = idesc_nvf4(attn::BM, attn::BN);
      const uint32_t sfk = tmem + T_SFK + 8 * b, sbuf = tmem + 128 * b;
      uint32_t t = 0, uc = 0, mine = 0, pc0 = 0;  // pc0: K stages (tile pairs) of the earlier units
      for (int i = 0, u = cta_unit(0, p.units); u >= 0; u = cta_unit(++i, p.units), ++uc) {
        const Unit un = unit_of(u, p);
        const int n = kv_tiles(un, p);
        const int qs = uc & 1;
        const uint8_t* qb = sm + OFF_Q + qs * Q_STAGE;
        const uint32_t sfq = tmem + T_SFQ + 8 * (2 * b + qs);
        int j = (int)(((uint32_t)b + NS - t % NS) % NS);  // this thread's first tile of the unit
        // every issuer waits for the unit's Q, tiles or not, so that its release below cannot count
        // toward the previous unit of the same Q stage
        mbar_wait(&q_full[qs], (uc >> 1) & 1, 0x703);
        if (j < n) {
          tc_fence_after();
          tmem_cp_sf_atom(sfq, smem_desc(smem_u32(qb + 8192), 16, 128, kSwizzleNone));
          tmem_cp_sf_atom(sfq + 4, smem_desc(smem_u32(qb + 8192 + 512), 16, 128, kSwizzleNone));
        }
        for (; j < n; j += NS, ++mine) {
          const uint32_t pc = pc0 + (uint32_t)(j >> 1);
          const int ks = (int)(pc % NK);
          const uint8_t* kb = sm + OFF_K + ks * K_STAGE + (j & 1) * 8192;      // this tile's codes
          const uint8_t* ka = sm + OFF_K + ks * K_STAGE + 16384 + (j & 1) * 1024;  // its scale atoms
          if (mine >= 1) mbar_wait(&s_free[b], (mine - 1) & 1, 0x704);
          mbar_wait(&k_full[ks], (pc / NK) & 1, 0x705);
          tc_fence_after();
          tmem_cp_sf_atom(sfk, smem_desc(smem_u32(ka), 16, 128, kSwizzleNone));
          tmem_cp_sf_atom(sfk + 4, smem_desc(smem_u32(ka + 512), 16, 128, kSwizzleNone));
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const uint64_t ad = smem_desc(smem_u32(kb) + kk * 32, 16, 512, kSwizzle64B);  // keys: M
            const uint64_t bd = smem_desc(smem_u32(qb) + kk * 32, 16, 512, kSwizzle64B);  // queries: N
            mma_nvf4(sbuf, ad, bd, idq, sfk + 4 * kk, sfq + 4 * kk, kk > 0 ? 1u : 0u);
          }
          tc_commit(&k_empty[ks]);
          if ((j & 1) == 0 && j == n - 1) tc_commit(&k_empty[ks]);  // a stage with one tile of the unit
          tc_commit(&s_full[b]);
        }
        tc_commit(&q_empty[qs]);  // every issuer, once per unit (after its last MMA of it, if any)
        t += n;
        pc0 += (uint32_t)(n + 1) >> 1;
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------- max warps
    const int quarter = warp & 3;            // TMEM lane quarter: keys 32*quarter .. +31 of a tile
    const int cb = (warp - 4) >> 2;          // query columns 32*cb .. +31
    const int lane = threadIdx.x & 31;
    const int key = quarter * 32 + lane;     // key within a tile
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const bool wlead = lane == 0;
    uint32_t t = 0, uc = 0;
    for (int i = 0, u = cta_unit(0, p.units); u >= 0; u = cta_unit(++i, p.units), ++uc) {
      const Unit un = unit_of(u, p);
      const int n = kv_tiles(un, p);
      float mx[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) mx[c] = -INFINITY;
      // this lane's key scale, from L2 (not shared memory, which the MMAs keep busy), one tile ahead
      const float* gkrow = p.gk + (int64_t)un.b * p.Tp + key;
      float gnext = __ldg(gkrow);
      for (int j = 0; j < n; ++j, ++t) {
        const int sb = (int)(t % NS);
        const float g = gnext;
        if (j + 1 < n) gnext = __ldg(gkrow + (j + 1) * attn::BN);
        // keys with index in tile > lim are masked (causal diagonal tile: lim = the query row)
        const bool diag = p.causal && j == un.qt;
        const int lim = p.T - 1 - j * attn::BN;
        mbar_wait(&s_full[sb], (t / NS) & 1, 0x706);
        tc_fence_after();
        uint32_t a[32];
        tmem_ld32(tmem + lane_base + 128 * sb + 32 * cb, a);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (wlead) mbar_arrive(&s_free[sb]);
        if (diag || key > lim) {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const bool masked = key > (diag ? 32 * cb + c : lim);
            mx[c] = masked ? mx[c] : fmaxf(mx[c], __fmul_rn(__uint_as_float(a[c]), g));
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) mx[c] = fmaxf(mx[c], __fmul_rn(__uint_as_float(a[c]), g));
        }
      }
      // max over this quarter's 32 keys for each of the 32 query columns: lane c holds column c
      const float m = warp_transpose_max(mx);
      float* st = stat + (uc & 1) * 512;
      st[quarter * 128 + 32 * cb + lane] = m;
      named_bar(1, 16 * 32);
      if (quarter == 0) {
        const int q = 32 * cb + lane;
        const float r = fmaxf(fmaxf(st[q], st[128 + q]), fmaxf(st[256 + q], st[384 + q]));
        p.row_max[((int64_t)un.b * p.HqT + p.hq0 + un.h) * p.Tp + un.qt * attn::BM + q] = r;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}
