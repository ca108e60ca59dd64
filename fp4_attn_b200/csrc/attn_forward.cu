// attn_forward.cu -- the FP4 attention forward as one C ABI call: the Q/K
// fake-quant operands, the V-hat planes and the attention kernel, with the
// packed operands in a caller-provided workspace (fp4attn_forward).
//
// This is the call a binding of the reference's patched attention makes
// (llama_patch.py:167-196 quantize Q/K/V, llama_patch.py:57-105 attend):
// bf16/fp16/fp32 [B,H,T,D] tensors with element strides in, fp32
// [B,T,Hq,D] out.
#include <stdint.h>

#include "fp4attn.h"
#include "status.h"

namespace {

constexpr int64_t kAlign = 256;

int64_t align_up(int64_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// offsets[0..7]: q codes, q scale atoms, q g, k codes, k scale atoms, k g,
// v hi, v lo.  Returns the total size, or -1 for a bad shape.
int64_t layout(int B, int Hq, int Hkv, int T, int D, int64_t* offsets) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || T <= 0 || D <= 0 || D % 64 != 0 || Hq % Hkv != 0) return -1;
  const int64_t Tp = ((int64_t)T + 127) / 128 * 128;
  const int64_t rows = (int64_t)B * Tp;
  const int64_t sz[8] = {
      rows * Hq * D / 2,                // q codes [B*Tp][Hq*D/2]
      rows / 128 * Hq * (D / 64) * 512,  // q tcgen05 scale atoms
      rows * 4,                          // q per-token g
      rows * Hkv * D / 2,
      rows / 128 * Hkv * (D / 64) * 512,
      rows * 4,
      (int64_t)B * Hkv * D * Tp * 2,  // v hi [B*Hkv*D][Tp] fp16
      (int64_t)B * Hkv * D * Tp * 2,  // v lo
  };
  int64_t off = 0;
  for (int i = 0; i < 8; ++i) {
    offsets[i] = off;
    off += align_up(sz[i]);
  }
  return off;
}

}  // namespace

extern "C" int64_t fp4attn_workspace_layout(int B, int Hq, int Hkv, int T, int D, int64_t* offsets) {
  int64_t tmp[8];
  return layout(B, Hq, Hkv, T, D, offsets ? offsets : tmp);
}

extern "C" int fp4attn_forward(const void* q, const void* k, const void* v, int in_dtype, int B, int Hq, int Hkv,
                               int T, int D, int64_t q_sB, int64_t q_sH, int64_t q_sT, int64_t k_sB, int64_t k_sH,
                               int64_t k_sT, int64_t v_sB, int64_t v_sH, int64_t v_sT, int causal, float scaling,
                               float* out, void* workspace, int64_t workspace_bytes, void* stream) {
  using namespace fp4;
  clear_error();
  if (!q || !k || !v || !out || !workspace) return set_error(FP4ATTN_ERR_ARG, "null pointer");
  if ((uintptr_t)workspace % kAlign) return set_error(FP4ATTN_ERR_ARG, "workspace must be 256-byte aligned");
  int64_t off[8];
  const int64_t need = layout(B, Hq, Hkv, T, D, off);
  if (need < 0) return set_error(FP4ATTN_ERR_ARG, "bad shape");
  if (workspace_bytes < need)
    return set_error(FP4ATTN_ERR_ARG, "workspace of %lld bytes, %lld needed", (long long)workspace_bytes,
                     (long long)need);
  const int Tp = (T + 127) / 128 * 128;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* qc = ws + off[0];
  uint8_t* qs = ws + off[1];
  float* gq = reinterpret_cast<float*>(ws + off[2]);
  uint8_t* kc = ws + off[3];
  uint8_t* ks = ws + off[4];
  float* gk = reinterpret_cast<float*>(ws + off[5]);
  uint16_t* vhi = reinterpret_cast<uint16_t*>(ws + off[6]);
  uint16_t* vlo = reinterpret_cast<uint16_t*>(ws + off[7]);
  // Q and K: row mode (per-token global scale) on the [B*T, H*D] views, tcgen05 scale atoms
  if (int e = fp4q_quantize(q, in_dtype, B, T, Hq, D, q_sB, q_sT, q_sH, Tp, 1, 0, 1536.0f, qc, (int64_t)Hq * D / 2,
                            qs, 1, (int64_t)Hq * D / 64, gq, nullptr, 0, 0, stream))
    return e;
  if (int e = fp4q_quantize(k, in_dtype, B, T, Hkv, D, k_sB, k_sT, k_sH, Tp, 1, 0, 1536.0f, kc,
                            (int64_t)Hkv * D / 2, ks, 1, (int64_t)Hkv * D / 64, gk, nullptr, 0, 0, stream))
    return e;
  if (int e = fp4attn_prepare_v(v, in_dtype, B, Hkv, T, D, v_sB, v_sH, v_sT, Tp, vhi, vlo, nullptr, nullptr, stream))
    return e;
  return fp4attn_fwd_packed(qc, qs, gq, kc, ks, gk, vhi, vlo, out, B, Hq, Hkv, T, Tp, D, causal, scaling, 0, stream);
}
