/*
 * nvfp4_oracle.c -- CPU restatement of the reference NVFP4 quantizer.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels in
 * fp4_attn_b200/csrc; it is linked only by tests/, __graft_entry__.smoke() and
 * the cpu_baseline / reference legs of bench.py.  Nothing in the product path
 * loads it.
 *
 * Two arithmetic flavours of the reference are restated here:
 *
 *  1. The torch path, FP4Quantizer.single_nvfp4_quant_dequant_fused
 *     (fp4_quant_utils.py:112-172), op for op, in the dequant dtype's
 *     arithmetic (fp32, bf16 or fp16: every torch op computes in fp32 and
 *     rounds once to the tensor dtype, which is what rnd() models):
 *        pad columns to a multiple of 16 with zeros               (:126-130)
 *        g = rowmax|x|  (aligned; no division by global_sf_max)   (:133-134)
 *        g = colmax|x| * recip(global_sf_max)  (not aligned)      (:135-139)
 *        x = x * recip(g)                                         (:141)
 *        s = e4m3(amax16|x| * recip(6))                           (:147-153)
 *        q = cast_to_fp4(clamp(x * recip(s), -6, 6))              (:158-160)
 *        out = (q * s) * g                                        (:161-165)
 *     recip(v) is get_reciprocal (:64-69): 0 where v == 0, else 1/v.
 *     cast_to_fp4 (:47-62) is round-half-to-even on the E2M1 grid with the
 *     sign taken from torch.sign, so -0.0 and NaN lose their sign there.
 *     The e4m3 cast is torch's float8_e4m3fn cast: RNE, |v| > 464 -> NaN.
 *
 *  2. The reference CUDA extension nvfp4sim (fast_fp4/nvfp4sim.cu):
 *        amax floor 1e-10, fmaxf (NaN ignored)                    (:104-113)
 *        scale byte = satfinite_e4m3((double)amax * (1.0/6.0))    (:116)
 *        candidate bytes b + lane - 7, wrapped to 8 bits (search) (:117)
 *        inv = (float)(1.0 / (double)scale)                       (:118-119)
 *        codes: clamp +-6, scale by 2^-126, add 1<<21, bits 22-24 (:76-85)
 *          = round-half-away-from-zero on the E2M1 grid
 *        loss = sum (deq*scale - x)^2, low 4 bits replaced by lane (:121-140)
 *        winner = minimum tagged loss                             (:142-153)
 *        decode: code bits -> float * 2^126, times the scale      (:87-94,292-307)
 *
 * Built by oracle/Makefile with -O2 -ffp-contract=off (no FMA contraction,
 * no fast-math: the E2M1 bit trick depends on fp32 denormals).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define ARITH_F32 0
#define ARITH_BF16 1
#define ARITH_F16 2

#define GMODE_NONE 0
#define GMODE_ROW 1
#define GMODE_COL 2

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* Round an fp32 value to bf16 (round to nearest even), returned widened. */
static inline float round_bf16(float v) {
    uint32_t u = f2u(v);
    if ((u & 0x7fffffffu) > 0x7f800000u) return u2f(u | 0x00400000u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return u2f(u & 0xffff0000u);
}

static inline float round_f16(float v) { return (float)(_Float16)v; }

/* One torch op in the dequant dtype: exact fp32 result rounded once. */
static inline float rnd(float v, int arith) {
    if (arith == ARITH_BF16) return round_bf16(v);
    if (arith == ARITH_F16) return round_f16(v);
    return v;
}

/* torch.max over |x|: NaN wins. */
static inline float nanmax(float a, float b) {
    if (isnan(a)) return a;
    if (isnan(b)) return b;
    return a > b ? a : b;
}

/* get_reciprocal (fp4_quant_utils.py:64-69) in the dequant dtype. */
static inline float recip(float v, int arith) {
    if (v == 0.0f) return 0.0f;
    return rnd(1.0f / v, arith);
}

/* ---------------------------------------------------------------- e4m3 */

/* Round a finite non-negative value onto the E4M3 grid (3 mantissa bits,
 * min normal exponent -6, subnormal step 2^-9), ties to even.  The result
 * may be 480 (one step above the largest finite value). */
static float e4m3_grid_rne(float a) {
    if (a == 0.0f) return 0.0f;
    int e;
    frexpf(a, &e);
    e -= 1; /* a = 1.f * 2^e */
    if (e < -6) e = -6;
    float step = ldexpf(1.0f, e - 3);
    float r = rintf(a / step); /* a/step is exact: division by a power of two */
    return r * step;
}

/* Encode an E4M3 value that lies on the grid (|v| <= 448) to its byte. */
static uint8_t e4m3_encode_exact(float v) {
    uint8_t sign = (f2u(v) >> 24) & 0x80u;
    float a = fabsf(v);
    if (a == 0.0f) return sign;
    if (a < 0.015625f) return sign | (uint8_t)(a * 512.0f); /* subnormal */
    int e;
    float f = frexpf(a, &e); /* a = f * 2^e, f in [0.5,1) */
    int ex = e - 1 + 7;
    int man = (int)((f * 2.0f - 1.0f) * 8.0f);
    return sign | (uint8_t)(ex << 3) | (uint8_t)man;
}

/* torch's float32 -> float8_e4m3fn cast (byte). */
uint8_t oracle_e4m3_from_f32_torch(float v) {
    uint8_t sign = (f2u(v) >> 24) & 0x80u;
    if (isnan(v)) return sign | 0x7fu;
    float r = e4m3_grid_rne(fabsf(v));
    if (r > 448.0f) return sign | 0x7fu; /* also covers inf */
    return sign | e4m3_encode_exact(r);
}

/* __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3) restated. */
uint8_t oracle_e4m3_from_f32_satfinite(float v) {
    uint8_t sign = (f2u(v) >> 24) & 0x80u;
    if (isnan(v)) return 0x7fu;
    float r = isinf(v) ? 448.0f : e4m3_grid_rne(fabsf(v));
    if (r > 448.0f) r = 448.0f;
    return sign | e4m3_encode_exact(r);
}

float oracle_e4m3_to_f32(uint8_t b) {
    float sign = (b & 0x80u) ? -1.0f : 1.0f;
    int ex = (b >> 3) & 15, man = b & 7;
    if (ex == 15 && man == 7) return u2f(((b & 0x80u) ? 0xffc00000u : 0x7fc00000u));
    if (ex == 0) return sign * (float)man * 0.001953125f;
    return sign * ldexpf(1.0f + (float)man / 8.0f, ex - 7);
}

/* ---------------------------------------------------------------- e2m1 */

static const float E2M1_VALUE[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

/* cast_to_fp4 magnitude step (fp4_quant_utils.py:53-60): grid index of |x|.
 * The reference applies eight torch.where passes in sequence; each later
 * pass only rewrites values the earlier ones left outside the grid, and
 * every grid value written lies outside the later passes' intervals, so
 * the sequence equals this single classification. */
static int e2m1_index_rne(float a) {
    if (a <= 0.25f) return 0;
    if (a < 0.75f) return 1;
    if (a <= 1.25f) return 2;
    if (a < 1.75f) return 3;
    if (a <= 2.5f) return 4;
    if (a < 3.5f) return 5;
    if (a <= 5.0f) return 6;
    return 7;
}

/* ------------------------------------------------ torch-path quantizer */

/*
 * oracle_fused_qdq: FP4Quantizer.single_nvfp4_quant_dequant_fused.
 *
 * x:       logical [m, n] input, element (i, j) at x[i*sm + j*sn]; the values
 *          are the input tensor's values widened to float (bf16/f16/f32).
 * gmode:   GMODE_NONE (global_sf_max=None), GMODE_ROW (aligned) or GMODE_COL.
 * arith:   the dequant dtype.
 * gsf_max: global_sf_max (col mode only).
 * Outputs (any may be NULL):
 *   out    [m, n]         dequantized values (in the dequant dtype, widened)
 *   codes  [m, npad/2]    E2M1 codes, element 2k in the low nibble
 *   scales [m, npad/16]   E4M3 block-scale bytes
 *   g      [m] (row) or [npad] (col): the global scale
 * Returns 0.
 */
int oracle_fused_qdq(const float* x, int64_t m, int64_t n, int64_t sm, int64_t sn,
                     int gmode, int arith, float gsf_max,
                     float* out, uint8_t* codes, uint8_t* scales, float* g) {
    const int64_t npad = (n + 15) / 16 * 16;
    const int64_t nblk = npad / 16;
    const float r6 = recip(6.0f, arith);
    const float rgsf = recip(rnd(gsf_max, arith), arith);
    float colg_local[1];
    float* colg = NULL;
    (void)colg_local;

    /* Column global scales need every row first. */
    if (gmode == GMODE_COL) {
        colg = g;
        for (int64_t j = 0; j < npad; ++j) colg[j] = 0.0f;
        for (int64_t i = 0; i < m; ++i)
            for (int64_t j = 0; j < n; ++j)
                colg[j] = nanmax(colg[j], fabsf(rnd(x[i * sm + j * sn], arith)));
        for (int64_t j = 0; j < npad; ++j) colg[j] = rnd(colg[j] * rgsf, arith);
    }

    float row[16];
    for (int64_t i = 0; i < m; ++i) {
        float gi = 0.0f;
        if (gmode == GMODE_ROW) {
            for (int64_t j = 0; j < n; ++j) gi = nanmax(gi, fabsf(rnd(x[i * sm + j * sn], arith)));
            if (g) g[i] = gi;
        }
        for (int64_t b = 0; b < nblk; ++b) {
            float amax = 0.0f;
            for (int k = 0; k < 16; ++k) {
                int64_t j = b * 16 + k;
                float v = (j < n) ? rnd(x[i * sm + j * sn], arith) : 0.0f;
                if (gmode == GMODE_ROW) v = rnd(v * recip(gi, arith), arith);
                else if (gmode == GMODE_COL) v = rnd(v * recip(colg[j], arith), arith);
                row[k] = v;
                amax = nanmax(amax, fabsf(v));
            }
            float s = rnd(amax * r6, arith);
            uint8_t sb = oracle_e4m3_from_f32_torch(s);
            s = oracle_e4m3_to_f32(sb); /* exact in every dequant dtype */
            float rs = recip(s, arith);
            if (scales) scales[i * nblk + b] = sb;
            for (int k = 0; k < 16; k += 2) {
                uint8_t nib[2];
                for (int t = 0; t < 2; ++t) {
                    int64_t j = b * 16 + k + t;
                    float v = rnd(row[k + t] * rs, arith);
                    /* torch.clamp keeps NaN */
                    if (!isnan(v)) v = v < -6.0f ? -6.0f : (v > 6.0f ? 6.0f : v);
                    float q;
                    uint8_t code;
                    if (isnan(v)) {
                        q = v;
                        code = 0;
                    } else {
                        int idx = e2m1_index_rne(fabsf(v));
                        /* torch.sign: +-0 -> 0, so q*sign is +0 for v = -0.0 */
                        float sgn = v > 0.0f ? 1.0f : (v < 0.0f ? -1.0f : 0.0f);
                        q = E2M1_VALUE[idx] * sgn;
                        code = (uint8_t)idx | ((f2u(q) >> 28) & 8u);
                    }
                    nib[t] = code;
                    float o = rnd(q * s, arith);
                    if (gmode == GMODE_ROW) o = rnd(o * gi, arith);
                    else if (gmode == GMODE_COL) o = rnd(o * colg[j], arith);
                    if (out && j < n) out[i * n + j] = o;
                }
                if (codes) codes[i * (npad / 2) + (b * 16 + k) / 2] = (uint8_t)(nib[0] | (nib[1] << 4));
            }
        }
    }
    return 0;
}

/* ------------------------------------------- reference CUDA extension */

/* f32_to_f4 (nvfp4sim.cu:76-85): two floats -> one byte, round half away. */
static uint8_t cuda_f32_to_f4(float a, float b) {
    const float scale = 1.1754943508222875e-38f; /* 2^-126 */
    a = fminf(fmaxf(-6.0f, a), 6.0f) * scale;
    b = fminf(fmaxf(-6.0f, b), 6.0f) * scale;
    uint32_t ua = f2u(a) + (1u << 21);
    uint32_t ub = f2u(b) + (1u << 21);
    ua = ((ua >> 22) & 7u) | ((ua >> 28) & 8u);
    ub = ((ub >> 22) & 7u) | ((ub >> 28) & 8u);
    return (uint8_t)(ua | (ub << 4));
}

/* f4_to_f32 (nvfp4sim.cu:87-94) for one nibble. */
static float cuda_f4_to_f32(uint32_t z) {
    const float iscale = 8.507059173023462e+37f; /* 2^126 */
    uint32_t u = ((z & 7u) << 22) | ((z & 8u) << 28);
    return u2f(u) * iscale;
}

/* One group of 16: the candidate loop of f32_to_nvf4_kernel (search=1) or
 * f32_to_nvf4_nosearch_kernel (search=0). */
static void cuda_quant_group(const float* x, int search, uint64_t* q_out, uint8_t* s_out) {
    float amax = 1e-10f;
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(x[i]));
    uint8_t base = oracle_e4m3_from_f32_satfinite((float)((double)amax * (1.0 / 6.0)));
    uint32_t best_tag = 0;
    int have = 0;
    for (int lane = 0; lane < 16; ++lane) {
        uint8_t sb = search ? (uint8_t)(base + (lane - 7)) : base;
        float sc = oracle_e4m3_to_f32(sb); /* via half in the reference: exact */
        float inv = (float)(1.0 / (double)sc);
        float loss = 0.0f;
        uint64_t q = 0;
        for (int i = 0; i < 8; ++i) {
            uint8_t byte = cuda_f32_to_f4(x[2 * i] * inv, x[2 * i + 1] * inv);
            q |= (uint64_t)byte << (8 * i);
            float d0 = cuda_f4_to_f32(byte & 15u) * sc - x[2 * i];
            float d1 = cuda_f4_to_f32(byte >> 4) * sc - x[2 * i + 1];
            loss += d0 * d0;
            loss += d1 * d1;
        }
        uint32_t tag = (f2u(loss) & ~15u) | (uint32_t)lane;
        float tagged = u2f(tag);
        /* fminf butterfly: NaN never wins while any lane is a number; among
         * numbers the smallest tagged value wins, so ties go to the lowest
         * lane for non-negative losses. */
        if (isnan(tagged)) continue;
        if (!have || tagged < u2f(best_tag)) {
            best_tag = tag;
            have = 1;
            *q_out = q;
            *s_out = sb;
        }
    }
}

/* f32_to_nvf4 / f32_to_nvf4_nosearch host + kernel (nvfp4sim.cu:96-192, 403-499).
 * Groups whose every candidate loss is NaN are left unwritten, as in the
 * reference (no lane matches the NaN minimum there). */
int oracle_cuda_f32_to_nvf4(uint64_t* xq, uint8_t* xs, const float* x, int64_t ngroups, int search) {
    for (int64_t gi = 0; gi < ngroups; ++gi) cuda_quant_group(x + gi * 16, search, xq + gi, xs + gi);
    return 0;
}

/* nvf4_to_f32 (nvfp4sim.cu:292-344). */
int oracle_cuda_nvf4_to_f32(float* out, const uint64_t* xq, const uint8_t* xs, int64_t ngroups) {
    for (int64_t gi = 0; gi < ngroups; ++gi) {
        float sc = oracle_e4m3_to_f32(xs[gi]);
        for (int i = 0; i < 16; ++i) out[gi * 16 + i] = cuda_f4_to_f32((uint32_t)(xq[gi] >> (4 * i)) & 15u) * sc;
    }
    return 0;
}

/* Decode torch-path codes/scales back to float (q*s), for tests. */
int oracle_decode_codes(float* out, const uint8_t* codes, const uint8_t* scales, int64_t m, int64_t npad) {
    for (int64_t i = 0; i < m; ++i)
        for (int64_t j = 0; j < npad; ++j) {
            uint8_t c = (codes[i * (npad / 2) + j / 2] >> (4 * (j & 1))) & 15u;
            float v = E2M1_VALUE[c & 7] * ((c & 8) ? -1.0f : 1.0f);
            out[i * npad + j] = v * oracle_e4m3_to_f32(scales[i * (npad / 16) + j / 16]);
        }
    return 0;
}
