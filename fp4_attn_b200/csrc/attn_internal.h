// attn_internal.h -- the attention kernel's launcher as the forward entry points
// call it (not part of the C ABI).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fp4 {

// Packed operands of one attention call and the KV heads it attends.  The
// operands hold all HqT query / HkvT KV heads of B batch rows (the
// [B*Tp, H*D] views the Q/K quantizer writes, V-hat planes [B*HkvT*D][Tp]);
// the call attends KV heads [hk0, hk1) with their query groups and writes
// out [B, T, (hk1 - hk0) * HqT / HkvT, D].
struct AttnLaunch {
  const uint8_t* q_codes;
  const uint8_t* q_scales;
  const float* q_g;
  const uint8_t* q_codes_lo;  // residual Q slice (dual-slice Q), or null
  const uint8_t* q_scales_lo;
  const float* q_g_lo;
  const uint8_t* k_codes;
  const uint8_t* k_scales;
  const float* k_g;
  const uint16_t* v_hi;
  const uint16_t* v_lo;
  void* out;
  float* row_max;  // scratch [B][HqT][Tp] fp32 for the row-maximum kernel, or null (max pass in the kernel)
  int B, HqT, HkvT, T, Tp, D;
  int hk0, hk1;
  int causal;
  float scaling;
  int flags;  // FP4ATTN_DUAL_P | FP4ATTN_OUT_BF16 | FP4ATTN_PV_FP16
  int num_ctas;
};

// Validates and launches fp4_attn_kernel on `st`; returns a status.
int launch_attention(const AttnLaunch& L, cudaStream_t st);

}  // namespace fp4
