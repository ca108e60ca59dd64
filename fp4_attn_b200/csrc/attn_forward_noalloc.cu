// attn_forward_noalloc.cu -- fp4attn_forward with a fixed, library-owned
// workspace: the call allocates no device memory.
//
// For callers that cannot hand the library device memory: a C or FFI binding
// with no device allocator of its own, or a serving loop that must not call
// cudaMalloc per request (it can synchronize the device and can fail under
// memory pressure mid-request).  The workspace is a file-scope __device__
// array of kNoAllocWorkspaceBytes; its address is looked up once per device
// (cudaGetSymbolAddress) on the first call made with that device current, so
// make that first call before any stream capture.  Every later call whose
// stream is not capturing looks the address up again: a device reset
// (cudaDeviceReset, or a reset of the primary context) reloads the module and
// the array can move, so only a call made during a capture uses the address
// the last call outside one found.
//
// Every call shares the one array: calls whose GPU work overlaps (different
// streams without ordering between them) race on it and corrupt each other's
// operands.  Issue them on one stream, or order them with events.
//
// Nothing in the array has to start at zero: each call writes every byte it
// later reads (padded rows of the Q/K operands are written as zeros by the
// quantizer, padded V-hat columns are cleared by fp4attn_prepare_v).
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "fp4attn.h"
#include "status.h"

namespace {

// 32 MiB: the Llama-3-8B attention shape (B=1, Hq=32, Hkv=8, T=4096, D=128)
// needs 27.3 MiB of packed operands.
constexpr int64_t kNoAllocWorkspaceBytes = 32ll << 20;
constexpr int kMaxDevices = 64;

std::atomic<void*> g_ws_ptr[kMaxDevices];  // per device: the array's address, once looked up

}  // namespace

// The fixed workspace (file scope, internal linkage).
static __device__ __align__(256) uint8_t g_noalloc_ws[kNoAllocWorkspaceBytes];

extern "C" int fp4attn_forward_noalloc(const void* q, const void* k, const void* v, int in_dtype, int B, int Hq,
                                       int Hkv, int T, int D, int64_t q_sB, int64_t q_sH, int64_t q_sT,
                                       int64_t k_sB, int64_t k_sH, int64_t k_sT, int64_t v_sB, int64_t v_sH,
                                       int64_t v_sT, int causal, float scaling, float* out, void* stream) {
  using namespace fp4;
  clear_error();
  const int64_t need = fp4attn_workspace_layout(B, Hq, Hkv, T, D, nullptr);
  if (need < 0) return set_error(FP4ATTN_ERR_ARG, "bad shape");
  if (need > kNoAllocWorkspaceBytes)
    return set_error(FP4ATTN_ERR_UNSUPPORTED,
                     "shape needs a %lld-byte workspace, above the fixed %lld bytes of fp4attn_forward_noalloc; "
                     "use fp4attn_forward with a caller workspace",
                     (long long)need, (long long)kNoAllocWorkspaceBytes);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(FP4ATTN_ERR_CUDA, "cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices) return set_error(FP4ATTN_ERR_UNSUPPORTED, "device index %d", dev);
  void* ws = g_ws_ptr[dev].load(std::memory_order_acquire);
  // a stream whose capture state cannot be read is treated as capturing
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  bool capturing = false;
  if (cudaStreamIsCapturing(reinterpret_cast<cudaStream_t>(stream), &cap) != cudaSuccess) {
    cudaGetLastError();
    capturing = true;
  } else {
    capturing = cap != cudaStreamCaptureStatusNone;
  }
  if (!ws || !capturing) {
    ws = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ws, g_noalloc_ws);
    if (e != cudaSuccess || !ws)
      return set_error(FP4ATTN_ERR_CUDA, "cudaGetSymbolAddress of the fixed workspace: %s", cudaGetErrorString(e));
    g_ws_ptr[dev].store(ws, std::memory_order_release);
  }
  return fp4attn_forward(q, k, v, in_dtype, B, Hq, Hkv, T, D, q_sB, q_sH, q_sT, k_sB, k_sH, k_sT, v_sB, v_sH, v_sT,
                         causal, scaling, out, ws, kNoAllocWorkspaceBytes, stream);
}
