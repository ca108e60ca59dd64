// status.h -- error reporting for the C ABI: every entry point returns a
// status code and keeps a per-thread message for fp4attn_last_error().
#pragma once

#include <cuda_runtime.h>

#define FP4ATTN_OK 0
#define FP4ATTN_ERR_ARG 1
#define FP4ATTN_ERR_CUDA 2
#define FP4ATTN_ERR_UNSUPPORTED 3

namespace fp4 {
void clear_error();
int set_error(int code, const char* fmt, ...);
// cudaGetLastError() after a launch, turned into a status.
int check_launch(const char* what);
// Count one kernel launch of this library (read by fp4attn_launch_count()).
void count_launch();
// Raise a kernel's dynamic shared memory limit to `bytes` (and allow non-portable
// cluster sizes when asked) on the current device.  Function attributes belong to
// each device's context, so this is done once per (kernel, device), under a lock;
// returns a status.
int set_smem_attr(const void* fn, int bytes, bool nonportable_cluster = false);
// Device status words of the translation units with bounded waits.
unsigned int gemm_status(bool reset);
unsigned int attn_status(bool reset);
unsigned int quant_status(bool reset);
unsigned int decode_status(bool reset);
unsigned int qkv_status(bool reset);
unsigned int peak_status(bool reset);
}  // namespace fp4
