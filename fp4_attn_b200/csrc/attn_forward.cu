// attn_forward.cu -- the FP4 attention forward as one C ABI call: the Q/K
// fake-quant operands, the V-hat planes and the attention kernel, with the
// packed operands in a caller-provided workspace (fp4attn_forward).
//
// This is the call a binding of the reference's patched attention makes
// (llama_patch.py:167-196 quantize Q/K/V, llama_patch.py:57-105 attend):
// bf16/fp16/fp32 [B,H,T,D] tensors with element strides in, fp32
// [B,T,Hq,D] out.
#include <stdint.h>

#include <stdio.h>

#include "attn_internal.h"
#include "fp4attn.h"
#include "status.h"

#include <algorithm>

#include "common.cuh"

namespace {

constexpr int64_t kAlign = 256;
constexpr int kPieces = 13;

int64_t align_up(int64_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// offsets[0..12]: q codes, q scale atoms, q g, k codes, k scale atoms, k g,
// v hi, v lo, then (dual-slice Q only, empty otherwise) the residual Q
// slice's codes, scale atoms and g, and an fp32 scratch [B*Tp][Hq*D] for
// Q - hi, then (single-slice Q only) the row maxima [B][Hq][Tp] fp32 of the
// row-maximum kernel.  Returns the total size, or -1 for a bad shape.
int64_t layout(int B, int Hq, int Hkv, int T, int D, int flags, int64_t* offsets) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || T <= 0 || D <= 0 || D % 64 != 0 || Hq % Hkv != 0) return -1;
  if (flags & ~(FP4ATTN_DUAL_Q | FP4ATTN_DUAL_P | FP4ATTN_OUT_BF16 | FP4ATTN_PV_FP16)) return -1;
  const int64_t Tp = ((int64_t)T + 127) / 128 * 128;
  const int64_t rows = (int64_t)B * Tp;
  const int64_t dq = (flags & FP4ATTN_DUAL_Q) ? 1 : 0;
  const int64_t sz[kPieces] = {
      rows * Hq * D / 2,                 // q codes [B*Tp][Hq*D/2]
      rows / 128 * Hq * (D / 64) * 512,  // q tcgen05 scale atoms
      rows * 4,                          // q per-token g
      rows * Hkv * D / 2,
      rows / 128 * Hkv * (D / 64) * 512,
      rows * 4,
      (int64_t)B * Hkv * D * Tp * 2,  // v hi [B*Hkv*D][Tp] fp16
      (int64_t)B * Hkv * D * Tp * 2,  // v lo
      dq * rows * Hq * D / 2,         // residual q slice
      dq * rows / 128 * Hq * (D / 64) * 512,
      dq * rows * 4,
      dq * rows * Hq * D * 4,  // Q - hi, fp32
      (1 - dq) * rows * Hq * 4,  // row maxima [B][Hq][Tp]
  };
  int64_t off = 0;
  for (int i = 0; i < kPieces; ++i) {
    offsets[i] = off;
    off += align_up(sz[i]);
  }
  return off;
}

// r = x - r on the [B*T, H*D] view of x [B,H,T,D] (r holds the first slice's
// dequantized values), zeros on the padding rows t >= T: the fp32 residual
// that dual_nvfp4 quantizes second (fp4_quant_utils.py:313-315).  Used when
// the one-pass dual quantizer does not take the layout.  One row per block
// iteration, columns across the threads (32-bit index math).
template <int DT>
__global__ void q_residual_kernel(const void* xv, int64_t sB, int64_t sT, int64_t sH, int B, int T, int Tp, int H,
                                  int D, float* r) {
  using Tin = typename fp4::In<DT>::T;
  const Tin* x = static_cast<const Tin*>(xv);
  const int hd = H * D, nrows = B * Tp;
  for (int row = blockIdx.x; row < nrows; row += gridDim.x) {
    const int b = row / Tp, t = row - b * Tp;
    float* rr = r + (int64_t)row * hd;
    const Tin* xr = x + (int64_t)b * sB + (int64_t)t * sT;
    for (int c = threadIdx.x; c < hd; c += blockDim.x) {
      const int h = c / D, d = c - h * D;
      rr[c] = t < T ? __fsub_rn(fp4::In<DT>::f(xr[(int64_t)h * sH + d]), rr[c]) : 0.0f;
    }
  }
}

int q_residual(const void* x, int in_dtype, int64_t sB, int64_t sT, int64_t sH, int B, int T, int Tp, int H, int D,
               float* r, cudaStream_t st) {
  const int threads = 256;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned grid = (unsigned)std::min<int64_t>((int64_t)B * Tp, (int64_t)sms * 8);
  switch (in_dtype) {
    case FP4_DT_F32: q_residual_kernel<FP4_DT_F32><<<grid, threads, 0, st>>>(x, sB, sT, sH, B, T, Tp, H, D, r); break;
    case FP4_DT_BF16: q_residual_kernel<FP4_DT_BF16><<<grid, threads, 0, st>>>(x, sB, sT, sH, B, T, Tp, H, D, r); break;
    case FP4_DT_F16: q_residual_kernel<FP4_DT_F16><<<grid, threads, 0, st>>>(x, sB, sT, sH, B, T, Tp, H, D, r); break;
    default: return fp4::set_error(FP4ATTN_ERR_ARG, "bad dtype");
  }
  return fp4::check_launch("q_residual_kernel");
}

// Two side streams and their fork/join events for the calling host thread on
// one device, created on first use (one set per thread, so concurrent callers
// never wait on each other's events).  nullptr if they cannot be created.
struct SideStreams {
  cudaStream_t s[2];
  cudaEvent_t fork, join[2];
};

SideStreams* side_streams() {
  constexpr int kMaxDev = 64;
  thread_local SideStreams tab[kMaxDev];
  thread_local signed char state[kMaxDev] = {};  // 0 untried, 1 ready, -1 failed
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
  if (state[dev] == 0) {
    SideStreams& t = tab[dev];
    bool ok = cudaStreamCreateWithFlags(&t.s[0], cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&t.s[1], cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreateWithFlags(&t.fork, cudaEventDisableTiming) == cudaSuccess &&
              cudaEventCreateWithFlags(&t.join[0], cudaEventDisableTiming) == cudaSuccess &&
              cudaEventCreateWithFlags(&t.join[1], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) cudaGetLastError();
    state[dev] = ok ? 1 : -1;
  }
  return state[dev] == 1 ? &tab[dev] : nullptr;
}

}  // namespace

extern "C" int64_t fp4attn_workspace_layout_ex(int B, int Hq, int Hkv, int T, int D, int flags, int64_t* offsets) {
  int64_t tmp[kPieces];
  return layout(B, Hq, Hkv, T, D, flags, offsets ? offsets : tmp);
}

extern "C" int64_t fp4attn_workspace_layout(int B, int Hq, int Hkv, int T, int D, int64_t* offsets) {
  int64_t tmp[kPieces];
  const int64_t n = layout(B, Hq, Hkv, T, D, 0, tmp);
  if (offsets)
    for (int i = 0; i < 8; ++i) offsets[i] = tmp[i];
  return n;
}

// Joins the side streams back into the caller's stream when it goes out of scope
// (every exit after the fork, error returns included): under stream capture an
// unjoined fork invalidates the caller's capture, and outside it the caller must
// not see the call return while side-stream kernels can still write its workspace.
struct SideJoin {
  SideStreams* side;
  cudaStream_t st;
  int join() {
    if (!side) return FP4ATTN_OK;
    SideStreams* sd = side;
    side = nullptr;
    if (cudaEventRecord(sd->join[0], sd->s[0]) != cudaSuccess || cudaEventRecord(sd->join[1], sd->s[1]) != cudaSuccess ||
        cudaStreamWaitEvent(st, sd->join[0], 0) != cudaSuccess || cudaStreamWaitEvent(st, sd->join[1], 0) != cudaSuccess)
      return fp4::set_error(FP4ATTN_ERR_CUDA, "stream join: %s", cudaGetErrorString(cudaGetLastError()));
    return FP4ATTN_OK;
  }
  ~SideJoin() {
    if (side) {
      char keep[512];  // an error already reported stays the reported one
      snprintf(keep, sizeof(keep), "%s", fp4attn_last_error());
      join();
      fp4::set_error(0, "%s", keep);
    }
  }
};

extern "C" int fp4attn_forward_heads(const void* q, const void* k, const void* v, int in_dtype, int B, int Hq, int Hkv,
                                     int T, int D, int64_t q_sB, int64_t q_sH, int64_t q_sT, int64_t k_sB,
                                     int64_t k_sH, int64_t k_sT, int64_t v_sB, int64_t v_sH, int64_t v_sT, int causal,
                                     float scaling, int flags, int hkv0, int hkv1, void* out, void* workspace,
                                     int64_t workspace_bytes, void* stream) {
  using namespace fp4;
  clear_error();
  if (!q || !k || !v || !out || !workspace) return set_error(FP4ATTN_ERR_ARG, "null pointer");
  if ((uintptr_t)workspace % kAlign) return set_error(FP4ATTN_ERR_ARG, "workspace must be 256-byte aligned");
  int64_t off[kPieces];
  const int64_t need = layout(B, Hq, Hkv, T, D, flags, off);
  if (need < 0) return set_error(FP4ATTN_ERR_ARG, "bad shape or flags");
  if (hkv0 < 0 || hkv1 > Hkv || hkv0 >= hkv1) return set_error(FP4ATTN_ERR_ARG, "bad KV-head range [%d, %d)", hkv0, hkv1);
  if (workspace_bytes < need)
    return set_error(FP4ATTN_ERR_ARG, "workspace of %lld bytes, %lld needed", (long long)workspace_bytes,
                     (long long)need);
  const int Tp = (T + 127) / 128 * 128;
  const bool dq = (flags & FP4ATTN_DUAL_Q) != 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* qc = ws + off[0];
  uint8_t* qs = ws + off[1];
  float* gq = reinterpret_cast<float*>(ws + off[2]);
  uint8_t* kc = ws + off[3];
  uint8_t* ks = ws + off[4];
  float* gk = reinterpret_cast<float*>(ws + off[5]);
  uint16_t* vhi = reinterpret_cast<uint16_t*>(ws + off[6]);
  uint16_t* vlo = reinterpret_cast<uint16_t*>(ws + off[7]);
  uint8_t* qc_lo = dq ? ws + off[8] : nullptr;
  uint8_t* qs_lo = dq ? ws + off[9] : nullptr;
  float* gq_lo = dq ? reinterpret_cast<float*>(ws + off[10]) : nullptr;
  float* qres = dq ? reinterpret_cast<float*>(ws + off[11]) : nullptr;
  float* row_max = dq ? nullptr : reinterpret_cast<float*>(ws + off[12]);
  const int64_t qld = (int64_t)Hq * D;
  // The three operand preparations are independent: K and V run on side streams
  // forked from and joined back to the caller's stream (capturable in a CUDA graph),
  // so the latency-bound K and V kernels overlap the Q quantization.  The Q/K/V
  // quantization always covers every head of the batch rows: the per-token global
  // scales span the whole [B*T, H*D] row (llama_patch.py:167-196), whatever heads
  // this call attends.
  SideStreams* side = side_streams();
  void* k_stream = stream;
  void* v_stream = stream;
  if (side && cudaEventRecord(side->fork, st) == cudaSuccess &&
      cudaStreamWaitEvent(side->s[0], side->fork, 0) == cudaSuccess &&
      cudaStreamWaitEvent(side->s[1], side->fork, 0) == cudaSuccess) {
    k_stream = side->s[0];
    v_stream = side->s[1];
  } else {
    cudaGetLastError();
    side = nullptr;
  }
  SideJoin joiner{side, st};
  if (int e = fp4q_quantize(k, in_dtype, B, T, Hkv, D, k_sB, k_sT, k_sH, Tp, 1, 0, 1536.0f, kc,
                            (int64_t)Hkv * D / 2, ks, 1, (int64_t)Hkv * D / 64, gk, nullptr, 0, 0, k_stream))
    return e;
  if (int e = fp4attn_prepare_v(v, in_dtype, B, Hkv, T, D, v_sB, v_sH, v_sT, Tp, vhi, vlo, nullptr, nullptr,
                                v_stream))
    return e;
  // Q and K: row mode (per-token global scale) on the [B*T, H*D] views, tcgen05 scale atoms.
  // Dual-slice Q: both slices in one pass over Q when the quantizer takes the layout; otherwise
  // the first slice's dequantized values go to the fp32 scratch, Q - hi is formed there and
  // quantized again (fp4_quant_utils.py:313-315).
  bool q_done = false;
  if (dq) {
    const int e = fp4q_quantize_dual(q, in_dtype, B, T, Hq, D, q_sB, q_sT, q_sH, Tp, qc, qld / 2, qs, 1, qld / 64, gq,
                                     qc_lo, qs_lo, gq_lo, stream);
    if (e != FP4ATTN_OK && e != FP4ATTN_ERR_UNSUPPORTED) return e;
    q_done = e == FP4ATTN_OK;
    clear_error();
  }
  if (!q_done) {
    if (int e = fp4q_quantize(q, in_dtype, B, T, Hq, D, q_sB, q_sT, q_sH, Tp, 1, 0, 1536.0f, qc, qld / 2, qs, 1,
                              qld / 64, gq, qres, dq ? FP4_DT_F32 : 0, dq ? qld : 0, stream))
      return e;
    if (dq) {
      if (int e = q_residual(q, in_dtype, q_sB, q_sT, q_sH, B, T, Tp, Hq, D, qres, st)) return e;
      if (int e = fp4q_quantize(qres, FP4_DT_F32, B, T, Hq, D, (int64_t)Tp * qld, qld, D, Tp, 1, 0, 1536.0f, qc_lo,
                                qld / 2, qs_lo, 1, qld / 64, gq_lo, nullptr, 0, 0, stream))
        return e;
    }
  }
  if (int e = joiner.join()) return e;
  AttnLaunch L{qc,  qs,      gq, qc_lo, qs_lo, gq_lo, kc, ks, gk,   vhi,  vlo,    out,
               row_max, B, Hq, Hkv,   T,     Tp,    D,  hkv0, hkv1, causal, scaling,
               flags & (FP4ATTN_DUAL_P | FP4ATTN_OUT_BF16 | FP4ATTN_PV_FP16), 0};
  return launch_attention(L, st);
}

extern "C" int fp4attn_forward_ex(const void* q, const void* k, const void* v, int in_dtype, int B, int Hq, int Hkv,
                                  int T, int D, int64_t q_sB, int64_t q_sH, int64_t q_sT, int64_t k_sB, int64_t k_sH,
                                  int64_t k_sT, int64_t v_sB, int64_t v_sH, int64_t v_sT, int causal, float scaling,
                                  int flags, void* out, void* workspace, int64_t workspace_bytes, void* stream) {
  return fp4attn_forward_heads(q, k, v, in_dtype, B, Hq, Hkv, T, D, q_sB, q_sH, q_sT, k_sB, k_sH, k_sT, v_sB, v_sH,
                               v_sT, causal, scaling, flags, 0, Hkv > 0 ? Hkv : 1, out, workspace, workspace_bytes,
                               stream);
}

extern "C" int fp4attn_forward(const void* q, const void* k, const void* v, int in_dtype, int B, int Hq, int Hkv,
                               int T, int D, int64_t q_sB, int64_t q_sH, int64_t q_sT, int64_t k_sB, int64_t k_sH,
                               int64_t k_sT, int64_t v_sB, int64_t v_sH, int64_t v_sT, int causal, float scaling,
                               float* out, void* workspace, int64_t workspace_bytes, void* stream) {
  return fp4attn_forward_ex(q, k, v, in_dtype, B, Hq, Hkv, T, D, q_sB, q_sH, q_sT, k_sB, k_sH, k_sT, v_sB, v_sH, v_sT,
                            causal, scaling, 0, out, workspace, workspace_bytes, stream);
}
