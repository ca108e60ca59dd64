/*
 * fp4attn.h -- C ABI of libfp4attn.so, the sm_100a NVFP4 quantizer and FP4
 * attention forward.
 *
 * Conventions for every entry point:
 *   - plain device pointers and sizes; `stream` is a cudaStream_t (NULL = the
 *     legacy default stream); work is enqueued asynchronously, nothing
 *     synchronizes;
 *   - outputs are caller-allocated and come first where the reference put
 *     them first; nothing is allocated on the device;
 *   - the return value is FP4ATTN_OK (0) or an error code, with a message
 *     for the calling thread in fp4attn_last_error().
 *
 * Dtype codes: 0 = float32, 1 = bfloat16, 2 = float16.
 */
#ifndef FP4ATTN_H
#define FP4ATTN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FP4ATTN_OK 0
#define FP4ATTN_ERR_ARG 1
#define FP4ATTN_ERR_CUDA 2
#define FP4ATTN_ERR_UNSUPPORTED 3

/* Message for the last failing call on this thread ("" when none). */
const char* fp4attn_last_error(void);
int fp4attn_version(void);
/* Number of kernels this library has launched in this process (all threads). */
unsigned long long fp4attn_launch_count(void);
/* Device-side status: 0, or the first bounded wait inside a kernel that gave
 * up ((site << 16) | (CTA index + 1)); such a kernel unwinds and returns
 * instead of hanging.  Synchronizes with the device; reset != 0 clears it. */
unsigned int fp4attn_device_status(int reset);

/* ------------------------------------------------------------------------
 * fp4_gemm_nvf4: C[m,n] = ga[m] * gb[n] * sum_k A[m,k] * B[n,k] on NVFP4
 * operands (tcgen05 kind::mxf4nvf4).  A and B are E2M1 codes [rows][ld]
 * bytes (K-major, two per byte, as fp4q_quantize writes them) with UE4M3
 * block scales in the tcgen05 atom layout (fp4q_quantize scale_layout 1);
 * ga/gb are per-row global scales or NULL.  C is fp32 [M][ldc].
 * K % 256 == 0.  No reference counterpart: the reference computes
 * attention scores with a dequantize + torch.matmul (llama_patch.py:71).
 * ---------------------------------------------------------------------- */
int fp4_gemm_nvf4(const uint8_t* a_codes, const uint8_t* a_scales, const float* a_g, const uint8_t* b_codes,
                  const uint8_t* b_scales, const float* b_g, float* c, int M, int N, int K, int64_t lda, int64_t ldb,
                  int64_t ldc, void* stream);

/* ------------------------------------------------------------------------
 * nvfp4sim module functions.  Each replaces one pybind11 binding of
 * fast_fp4/wrapper.cpp:41-45 (host functions fast_fp4/nvfp4sim.cu:156, 463,
 * 254, 309, 365) with the same argument order and meaning: `ngroups` groups
 * of 16 values, ngroups even; codes are 16 E2M1 nibbles per uint64 (element
 * i in bits 4i..4i+3), scales one E4M3 byte per group.  The reference's
 * numerics are kept: 1e-10 amax floor, satfinite scale, round-half-away E2M1
 * encode, and (search variants) the 16-candidate scale search.
 * ---------------------------------------------------------------------- */

/* nvfp4sim.f32_to_nvf4 (fast_fp4/wrapper.cpp:41, nvfp4sim.cu:156-192). */
int nvfp4sim_f32_to_nvf4(uint64_t* xq_out, uint8_t* xs_out, const float* x_in, int64_t ngroups, void* stream);

/* nvfp4sim.f32_to_nvf4_nosearch (fast_fp4/wrapper.cpp:42, nvfp4sim.cu:463-499). */
int nvfp4sim_f32_to_nvf4_nosearch(uint64_t* xq_out, uint8_t* xs_out, const float* x_in, int64_t ngroups,
                                  void* stream);

/* nvfp4sim.f16_to_nvf4 (fast_fp4/wrapper.cpp:44, nvfp4sim.cu:254-289); x_in holds IEEE halves. */
int nvfp4sim_f16_to_nvf4(uint64_t* xq_out, uint8_t* xs_out, const uint16_t* x_in, int64_t ngroups, void* stream);

/* nvfp4sim.nvf4_to_f32 (fast_fp4/wrapper.cpp:43, nvfp4sim.cu:309-344). */
int nvfp4sim_nvf4_to_f32(float* x_out, const uint64_t* xq_in, const uint8_t* xs_in, int64_t ngroups, void* stream);

/* nvfp4sim.nvf4_to_f16 (fast_fp4/wrapper.cpp:45, nvfp4sim.cu:365-400). */
int nvfp4sim_nvf4_to_f16(uint16_t* x_out, const uint64_t* xq_in, const uint8_t* xs_in, int64_t ngroups,
                         void* stream);

/* ------------------------------------------------------------------------
 * fp4q_quantize: block-16 NVFP4 quantize and (optionally) dequantize,
 * bit-exact to FP4Quantizer.single_nvfp4_quant_dequant_fused
 * (fp4_quant_utils.py:112-172), which it replaces, together with the torch
 * glue of single_nvfp4 (fp4_quant_utils.py:336-341).
 *
 * Input: logical matrix with row (b, t) and column c = h*D + d, element at
 * x[b*sB + t*sT + h*sH + d] (element strides; d contiguous).  A plain 2-D
 * [m, n] tensor is B=1, T=m, H=1, D=n, sT=n.  Columns are padded with zeros
 * to a multiple of 16 (fp4_quant_utils.py:126-130).
 *
 * gmode: 0 none (global_sf_max=None), 1 row (global_scale_aligned=True:
 *   g = rowmax|x|, not divided by global_sf_max), 2 column (aligned=False:
 *   g = colmax|x| * recip(global_sf_max); needs H == 1), 3 tensor
 *   (g = max|x| * recip(global_sf_max), then the row-mode formulas).
 * arith: the dequant dtype whose arithmetic is reproduced (0/1/2).
 *
 * Outputs (each optional, NULL to skip), output row index o = b*T_pad + t;
 * rows with t >= T are written as zeros:
 *   codes  [o][codes_ld] bytes, element 2k in the low nibble of byte k;
 *   scales E4M3 bytes; scale_layout 0: linear [o][scales_ld];
 *          scale_layout 1: tcgen05 block-scaled MMA atoms (128 rows x 4
 *          blocks, 512 bytes, k-fastest), scales_ld = blocks-per-row / 4
 *          rounded up;
 *   g      row: [B*T_pad]; column: [npad]; tensor: [1] (in/out workspace of
 *          the reduction; required when gmode != 0);
 *   out    dequantized values [o][out_ld] in out_dtype.
 * gmode | 0x10 (column and tensor modes): g already holds the global
 *   scale(s) (from fp4q_global_scale or a calibration), skip the reduction.
 * ---------------------------------------------------------------------- */
int fp4q_quantize(const void* x, int in_dtype, int B, int T, int H, int D, int64_t sB, int64_t sT, int64_t sH,
                  int T_pad, int gmode, int arith, float global_sf_max, uint8_t* codes, int64_t codes_ld,
                  uint8_t* scales, int scale_layout, int64_t scales_ld, float* g, void* out, int out_dtype,
                  int64_t out_ld, void* stream);

/* Dual-slice row mode in one pass (dual_nvfp4 without search,
 * fp4_quant_utils.py:307-315, on the row-aligned quantizer): slice 1 as
 * fp4q_quantize gmode 1 (fp32 arithmetic) into codes / scales / g, slice 2 =
 * the same quantizer on the fp32 residual x - dequant(slice 1) into codes_lo /
 * scales_lo / g_lo (same layouts).  Returns FP4ATTN_ERR_UNSUPPORTED for
 * layouts the one-pass kernel does not take (rows not 16-byte aligned, more
 * than 8192 columns); fp4q_quantize with an fp32 out then does the same in
 * three steps. */
int fp4q_quantize_dual(const void* x, int in_dtype, int B, int T, int H, int D, int64_t sB, int64_t sT, int64_t sH,
                       int T_pad, uint8_t* codes, int64_t codes_ld, uint8_t* scales, int scale_layout,
                       int64_t scales_ld, float* g, uint8_t* codes_lo, uint8_t* scales_lo, float* g_lo, void* stream);

/* The global-scale reduction of fp4q_quantize alone (gmode 2: column, 3:
 * tensor): g = max|x| * recip(global_sf_max) in the dequant dtype, written to
 * g ([npad] or [1]).  Same input description as fp4q_quantize.  Replaces the
 * torch.max/abs/get_reciprocal steps of fp4_quant_utils.py:135-139. */
int fp4q_global_scale(const void* x, int in_dtype, int B, int T, int H, int D, int64_t sB, int64_t sT, int64_t sH,
                      int gmode, int arith, float global_sf_max, float* g, void* stream);

/* ------------------------------------------------------------------------
 * FP4 attention forward: the native replacement for eager_attention_forward
 * with FP4 fake-quant (llama_patch.py:57-105) fed by the Q/K/V fake-quant of
 * llama_patch.py:167-196.  Three calls:
 *   1. fp4q_quantize on Q and K ([B,H,T,D] viewed as [B*T, H*D], row mode,
 *      T_pad = Tp, scale_layout 1) -> codes [B*Tp][H*D/2], scale atoms,
 *      per-token g [B*Tp];
 *   2. fp4attn_prepare_v on V;
 *   3. fp4attn_fwd_packed.
 * Tp = T rounded up to a multiple of 128.
 * ---------------------------------------------------------------------- */

/* V -> Vhat = single_nvfp4(v2d.T, global_scale_aligned=False) in fp32
 * arithmetic (llama_patch.py:196, fp4_quant_utils.py:112-172), stored as
 * fp16 hi/lo planes [B*Hkv*D][Tp] (row (b*Hkv+h)*D+d, column t; hi+lo keeps
 * 22 significant bits of Vhat, |Vhat| < 65504).  v is [B,Hkv,T,D] with
 * element strides sB, sH, sT and d contiguous.  vhat (fp32, same layout) and
 * g ([B*T], per-token global scale) are optional outputs.  Hkv*D <= 6144
 * (bf16 / fp16 input) or 3072 (fp32 input). */
int fp4attn_prepare_v(const void* v, int in_dtype, int B, int Hkv, int T, int D, int64_t sB, int64_t sH, int64_t sT,
                      int Tp, uint16_t* v_hi, uint16_t* v_lo, float* vhat, float* g, void* stream);

/* O[b,t,hq,:] = sum_j Phat[t,j] Vhat[j,:] with S = Qhat Khat^T * scaling,
 * causal or not, GQA (Hq % Hkv == 0), Phat = NVFP4 fake-quant of softmax(S)
 * per row (llama_patch.py:81-99).  out is fp32 [B,T,Hq,D].  D = 128.
 * num_ctas 0 = one persistent CTA per SM. */
int fp4attn_fwd_packed(const uint8_t* q_codes, const uint8_t* q_scales, const float* q_g, const uint8_t* k_codes,
                       const uint8_t* k_scales, const float* k_g, const uint16_t* v_hi, const uint16_t* v_lo,
                       float* out, int B, int Hq, int Hkv, int T, int Tp, int D, int causal, float scaling,
                       int num_ctas, void* stream);

/* fp4attn_fwd_packed with the reference's dual-slice options
 * (fp4_quant_utils.py:307-315 dual_nvfp4; FP4_USE_DUAL_QUANT_Q at
 * llama_patch.py:183-189 and FP4_USE_DUAL_QUANT_ATTN at llama_patch.py:84-95,
 * both default true in the reference).  q_codes_lo / q_scales_lo / q_g_lo:
 * the second (residual) Q slice, the same quantizer on Q - dequant(first
 * slice), same layouts; NULL = single-slice Q.  flags: FP4ATTN_DUAL_P for
 * P-hat = hi + lo with lo the row-aligned NVFP4 fake-quant of P - hi (one
 * more pass over the keys finds each row's residual scale); FP4ATTN_OUT_BF16
 * for a bf16 out (the reference's output dtype, llama_patch.py:102-103),
 * else fp32. */
int fp4attn_fwd_packed_dual(const uint8_t* q_codes, const uint8_t* q_scales, const float* q_g,
                            const uint8_t* q_codes_lo, const uint8_t* q_scales_lo, const float* q_g_lo,
                            const uint8_t* k_codes, const uint8_t* k_scales, const float* k_g, const uint16_t* v_hi,
                            const uint16_t* v_lo, void* out, int B, int Hq, int Hkv, int T, int Tp, int D,
                            int causal, float scaling, int flags, int num_ctas, void* stream);

/* fp4attn_fwd_packed_dual on operands holding Hq / Hkv heads, attending only
 * KV heads [hkv0, hkv1) and their query groups; out [B, T, (hkv1 - hkv0) *
 * Hq / Hkv, D].  The kernel step of fp4attn_forward_heads.  row_max: a
 * [B][Hq][Tp] fp32 scratch (16-byte aligned) for single-slice Q -- the row
 * maxima of the scores then come from a separate row-maximum kernel and the
 * attention kernel reads every K tile once; NULL keeps the kernel's own max
 * pass.  flags also takes FP4ATTN_PV_FP16. */
int fp4attn_fwd_packed_heads(const uint8_t* q_codes, const uint8_t* q_scales, const float* q_g,
                             const uint8_t* q_codes_lo, const uint8_t* q_scales_lo, const float* q_g_lo,
                             const uint8_t* k_codes, const uint8_t* k_scales, const float* k_g, const uint16_t* v_hi,
                             const uint16_t* v_lo, float* row_max, void* out, int B, int Hq, int Hkv, int T, int Tp,
                             int D, int hkv0, int hkv1, int causal, float scaling, int flags, void* stream);

/* Workspace of fp4attn_forward for a shape: writes the byte offsets of its
 * eight pieces -- Q codes, Q scale atoms, Q g, K codes, K scale atoms, K g,
 * V-hat hi plane, V-hat lo plane, each 256-byte aligned, laid out as steps 1
 * and 2 above describe -- to offsets[0..7] (may be NULL) and returns the
 * total size in bytes; -1 for a bad shape.  No reference counterpart: the
 * reference materialises the fake-quantized tensors in torch instead. */
int64_t fp4attn_workspace_layout(int B, int Hq, int Hkv, int T, int D, int64_t* offsets);

/* Flags of fp4attn_forward_ex / fp4attn_workspace_layout_ex. */
#define FP4ATTN_DUAL_Q 1 /* dual-slice Q (FP4_USE_DUAL_QUANT_Q=true) */
#define FP4ATTN_DUAL_P 2 /* dual-slice P (FP4_USE_DUAL_QUANT_ATTN=true) */
#define FP4ATTN_OUT_BF16 4 /* out is bf16 [B,T,Hq,D] (the reference's output dtype), not fp32 */
/* PV reads V-hat rounded once to fp16 for every query tile but the first 128
 * queries of each sequence (which keep the exact hi + lo planes): half the
 * PV tensor work.  Max-abs 2.7e-3 x RMS(O), cosine 0.99999999 against the
 * exact V-hat on the Llama-3-8B attention shape (1.4e-3 on the long-context
 * prefill inputs); without it PV is exact. */
#define FP4ATTN_PV_FP16 8

/* fp4attn_workspace_layout with flags: offsets[0..12], the eight pieces
 * above, then (FP4ATTN_DUAL_Q only; empty otherwise) the residual Q slice's
 * codes, scale atoms and g, and an fp32 [B*Tp][Hq*D] scratch, then (single-
 * slice Q only) the row maxima [B][Hq][Tp] fp32 of the row-maximum kernel. */
int64_t fp4attn_workspace_layout_ex(int B, int Hq, int Hkv, int T, int D, int flags, int64_t* offsets);

/* Steps 1-3 as one call: q [B,Hq,T,D], k and v [B,Hkv,T,D] in in_dtype
 * (FP4_DT_F32 / BF16 / F16) with element strides (sB, sH, sT) each and d
 * contiguous; out fp32 [B,T,Hq,D]; the packed operands go to workspace
 * (256-byte aligned, at least fp4attn_workspace_layout bytes).  Replaces the
 * Q/K/V fake-quant of llama_patch.py:167-196 plus eager_attention_forward
 * with P fake-quant (llama_patch.py:57-105). */
int fp4attn_forward(const void* q, const void* k, const void* v, int in_dtype, int B, int Hq, int Hkv, int T, int D,
                    int64_t q_sB, int64_t q_sH, int64_t q_sT, int64_t k_sB, int64_t k_sH, int64_t k_sT, int64_t v_sB,
                    int64_t v_sH, int64_t v_sT, int causal, float scaling, float* out, void* workspace,
                    int64_t workspace_bytes, void* stream);

/* fp4attn_forward with flags (FP4ATTN_DUAL_Q, FP4ATTN_DUAL_P): the reference's
 * dual-slice Q and / or P.  workspace: fp4attn_workspace_layout_ex(..., flags)
 * bytes.  With FP4ATTN_DUAL_Q the second Q slice is the row-mode quantizer on
 * the fp32 residual Q - dequant(first slice), bit-exact to dual_nvfp4. */
int fp4attn_forward_ex(const void* q, const void* k, const void* v, int in_dtype, int B, int Hq, int Hkv, int T, int D,
                       int64_t q_sB, int64_t q_sH, int64_t q_sT, int64_t k_sB, int64_t k_sH, int64_t k_sT,
                       int64_t v_sB, int64_t v_sH, int64_t v_sT, int causal, float scaling, int flags, void* out,
                       void* workspace, int64_t workspace_bytes, void* stream);

/* fp4attn_forward_ex attending only KV heads [hkv0, hkv1) and their query
 * groups: the shard of one rank when a job is split by (batch, KV head).  The
 * Q/K/V fake-quant still runs on every head of the B batch rows given (the
 * reference's per-token global scales span the whole [B*T, H*D] row,
 * llama_patch.py:167-196), so the packed operands -- and therefore every
 * attended head's output -- equal the unsharded call's bit for bit.  out is
 * [B, T, (hkv1 - hkv0) * Hq / Hkv, D]; workspace as fp4attn_forward_ex. */
int fp4attn_forward_heads(const void* q, const void* k, const void* v, int in_dtype, int B, int Hq, int Hkv, int T,
                          int D, int64_t q_sB, int64_t q_sH, int64_t q_sT, int64_t k_sB, int64_t k_sH, int64_t k_sT,
                          int64_t v_sB, int64_t v_sH, int64_t v_sT, int causal, float scaling, int flags, int hkv0,
                          int hkv1, void* out, void* workspace, int64_t workspace_bytes, void* stream);

/* fp4attn_forward without a caller workspace; allocates no device memory.
 * No counterpart in the reference.  For callers that cannot hand the library
 * device memory: a C/FFI binding without a device allocator of its own, or a
 * serving loop that must not call cudaMalloc per request (it can synchronize
 * the device and fail under memory pressure).  The packed operands live in a
 * fixed library-owned device array of 32 MiB (33554432 bytes); shapes whose
 * fp4attn_workspace_layout size exceeds it are rejected with
 * FP4ATTN_ERR_UNSUPPORTED.  The array's address is looked up on the first
 * call per device, so make that call before any stream capture; later calls
 * look it up again whenever `stream` is not capturing (a device reset
 * reloads the library's device code, and the array can move), and a call
 * made during a capture uses the address of the last call outside one.  All calls
 * share the array: calls whose GPU work overlaps race; issue them on one
 * stream or order them with events.  Nothing has to start zeroed. */
int fp4attn_forward_noalloc(const void* q, const void* k, const void* v, int in_dtype, int B, int Hq, int Hkv, int T,
                            int D, int64_t q_sB, int64_t q_sH, int64_t q_sT, int64_t k_sB, int64_t k_sH, int64_t k_sT,
                            int64_t v_sB, int64_t v_sH, int64_t v_sT, int causal, float scaling, float* out,
                            void* stream);

/* ------------------------------------------------------------------------
 * Q or K projection fused with RoPE and the NVFP4 row quantizer: the packed
 * attention operand straight from the hidden states.  Replaces q_proj/k_proj
 * (llama_patch.py:147-149), the row-wise fake-quant of the [B*T, H*D] view
 * (llama_patch.py:167-194) and the rotation (llama_patch.py:210), with the
 * rotation applied before the quantization (HF apply_rotary_pos_emb in bf16,
 * op for op).  x: bf16 [M][K] hidden states (M = B*T tokens), w: bf16
 * [H*128][K] (the nn.Linear weight), cos / sin: bf16 [M][128] per token.
 * Writes codes [M][H*64], E4M3 scales in tcgen05 atoms (H*2 groups per
 * 128-row block, the layout fp4attn_fwd_packed reads) and g [M].  T % 128 ==
 * 0, M % T == 0, K % 32 == 0, H = 1, 2 or a multiple of 4 up to 64; 16-byte
 * aligned buffers.  Two memsets (g, and 8 code bytes per 128-token block
 * that serve as the block's hand-off words until the kernel writes them) and
 * one cooperative launch of at most one CTA per SM; needs a device with
 * cooperative launch. */
int fp4qkv_rope_quant(const void* x, const void* w, const void* cos, const void* sin, int M, int K, int H, int T,
                      uint8_t* codes, uint8_t* scales, float* g, void* stream);

/* ------------------------------------------------------------------------
 * Decode: one new query token per sequence over an NVFP4 KV cache.  The
 * reference appends each call's fake-quantized K/V to the HF cache
 * (llama_patch.py:167-215) and attends over every cached key with P
 * fake-quant (llama_patch.py:57-105); the cache here holds the packed data
 * of those values (fp4_attn_b200.kv_cache.NVFP4KVCache):
 *   k_codes [B][Hkv][Tmax][D/2], k_scales E4M3 [B][Hkv][Tmax][D/16],
 *   k_g [B][Tmax] (per-token row-mode global scale);
 *   V dim-major: v_codes [B][Hkv][D][Tmax/2] (byte j of a channel holds
 *   tokens 2j, low nibble, and 2j+1), v_scales E4M3 [B][Hkv][D][Tmax] (one per
 *   element: V's blocks run along the tokens of the call that appended them),
 *   v_g [B][Tmax].
 * The query is packed the same way, row mode on its [B, Hq*D] view:
 * q_codes [B][Hq*D/2], q_scales E4M3 [B][Hq*D/16], q_g [B]; out fp32 [B][Hq][D];
 * len cached tokens are attended (no mask: the query is the newest token).
 * D = 128, Hq/Hkv <= 16, Tmax a multiple of 256 (the kernels copy whole
 * chunks of 256 keys; keys past len are read but not used).  The cache
 * buffers, g arrays and workspace are 16-byte aligned.  workspace:
 * fp4attn_decode_workspace_size bytes, nothing has to start zeroed. */
int64_t fp4attn_decode_workspace_size(int B, int Hq, int len);
int fp4attn_decode(const uint8_t* q_codes, const uint8_t* q_scales, const float* q_g, const uint8_t* k_codes,
                   const uint8_t* k_scales, const float* k_g, const uint8_t* v_codes, const uint8_t* v_scales,
                   const float* v_g, int B, int Hq, int Hkv, int D, int len, int Tmax, float scaling, float* out,
                   void* workspace, int64_t workspace_bytes, void* stream);
/* fp4attn_decode with V's scales also stored once per 16-token group for a
 * prefix of the cache: v_scales16 E4M3 [B][Hkv][D][Tmax/16], valid for the
 * first len16 tokens (a multiple of 16, <= len; 0 and NULL = none), whose
 * groups each came from one quantization block (a call that started on a group
 * boundary with whole blocks per sequence).  Chunks of 256 keys inside the
 * prefix read these instead of v_scales (2 KB instead of 32 KB per chunk and
 * KV head); the result is identical. */
int fp4attn_decode_ex(const uint8_t* q_codes, const uint8_t* q_scales, const float* q_g, const uint8_t* k_codes,
                      const uint8_t* k_scales, const float* k_g, const uint8_t* v_codes, const uint8_t* v_scales,
                      const float* v_g, const uint8_t* v_scales16, int len16, int B, int Hq, int Hkv, int D, int len,
                      int Tmax, float scaling, float* out, void* workspace, int64_t workspace_bytes, void* stream);

/* Measurement aid, no reference counterpart: one CTA per SM (num_ctas <= 0)
 * issues `iters` pairs of back-to-back tcgen05.mma.kind::mxf4nvf4 (M=128,
 * N=128, K=64 each) on fixed pseudo-random NVFP4 operands: the dense NVFP4
 * tensor throughput the FP4 contractions are measured against.  FLOPs per
 * launch = ctas * iters * 4194304; time the launch with events on `stream`.
 * iters <= 2^20. */
int fp4_mma_peak_run(int iters, int num_ctas, void* stream);

/* Profiling aid: a non-NULL buf makes later fp4attn_fwd_packed calls record
 * an event timeline (SM clock cycles from clock64) of each CTA's first work unit into
 * buf[cta * 512 + slot] (grid * 512 int64 entries); NULL turns it off. */
void fp4attn_set_trace(long long* buf);

#ifdef __cplusplus
}
#endif

#endif /* FP4ATTN_H */
