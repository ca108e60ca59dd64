// quant_f16.cu -- quantizer kernels instantiated for f16 input.
#include "quant_impl.cuh"

namespace fp4 {
int quant_dispatch_f16(const QuantArgs& p, int arith, int out_dtype, float* g, float gsf_max, int what,
                        cudaStream_t st) {
  return dispatch_arith<FP4_DT_F16>(p, arith, out_dtype, g, gsf_max, what, st);
}
int quant_dual_f16(const QuantArgs& p, cudaStream_t st) { return launch_rows_dual<FP4_DT_F16>(p, st); }
}  // namespace fp4
