// status.cu -- per-thread error message storage and library identity.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>
#include <vector>

#include "status.h"

namespace fp4 {

static thread_local char g_msg[512];

void clear_error() { g_msg[0] = 0; }

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

static unsigned long long g_launches = 0;

void count_launch() { __atomic_add_fetch(&g_launches, 1ull, __ATOMIC_RELAXED); }

int set_smem_attr(const void* fn, int bytes, bool nonportable_cluster) {
  struct Done {
    const void* fn;
    int dev, bytes;
  };
  static std::mutex mu;
  static std::vector<Done> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(FP4ATTN_ERR_CUDA, "cudaGetDevice failed");
  std::lock_guard<std::mutex> lock(mu);
  for (const Done& d : done)
    if (d.fn == fn && d.dev == dev && d.bytes >= bytes) return FP4ATTN_OK;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && nonportable_cluster)
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(FP4ATTN_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  }
  done.push_back({fn, dev, bytes});
  return FP4ATTN_OK;
}

int check_launch(const char* what) {
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FP4ATTN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return FP4ATTN_OK;
}

}  // namespace fp4

extern "C" const char* fp4attn_last_error(void) { return fp4::g_msg; }

extern "C" int fp4attn_version(void) { return 1; }

// Synchronizes with the device (reads device symbols).  Non-zero means a
// bounded wait inside a kernel gave up: (site << 16) | (CTA index + 1).
extern "C" unsigned int fp4attn_device_status(int reset) {
  // first non-zero status of the kernels with bounded waits; every word is read (and reset if asked)
  const unsigned int s[6] = {fp4::gemm_status(reset != 0),   fp4::attn_status(reset != 0),
                             fp4::quant_status(reset != 0),  fp4::decode_status(reset != 0),
                             fp4::qkv_status(reset != 0),    fp4::peak_status(reset != 0)};
  for (unsigned int v : s)
    if (v) return v;
  return 0;
}

extern "C" unsigned long long fp4attn_launch_count(void) { return __atomic_load_n(&fp4::g_launches, __ATOMIC_RELAXED); }
