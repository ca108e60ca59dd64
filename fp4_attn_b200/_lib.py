"""ctypes binding of libfp4attn.so (the C ABI declared in include/fp4attn.h).

The library is the only compute path: if it is missing, or no CUDA device is
visible, calls raise -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libfp4attn.so")

DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_lib = None

# Every exported entry point: name -> (argtypes, restype).
_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float
SIGNATURES = {
    "fp4attn_last_error": ([], ctypes.c_char_p),
    "fp4attn_version": ([], _I),
    "fp4attn_launch_count": ([], ctypes.c_ulonglong),
    "fp4attn_device_status": ([_I], ctypes.c_uint),
    "fp4_gemm_nvf4": ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _L, _L, _L, _P], _I),
    "fp4attn_set_trace": ([_P], None),
    "fp4_mma_peak_run": ([_I, _I, _P], _I),
    "fp4attn_prepare_v": ([_P, _I, _I, _I, _I, _I, _L, _L, _L, _I, _P, _P, _P, _P, _P], _I),
    "fp4attn_fwd_packed": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _I, _P], _I),
    "fp4attn_workspace_layout": ([_I, _I, _I, _I, _I, _P], _L),
    "fp4q_quantize_dual": ([_P, _I, _I, _I, _I, _I, _L, _L, _L, _I, _P, _L, _P, _I, _L, _P, _P, _P, _P, _P], _I),
    "fp4qkv_rope_quant": ([_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P], _I),
    "fp4attn_workspace_layout_ex": ([_I, _I, _I, _I, _I, _I, _P], _L),
    "fp4attn_fwd_packed_dual": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _I, _I,
                                 _P], _I),
    "fp4attn_fwd_packed_heads": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I,
                                  _I, _F, _I, _P], _I),
    "fp4attn_decode_workspace_size": ([_I, _I, _I], _L),
    "fp4attn_decode": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _P, _P, _L, _P], _I),
    "fp4attn_decode_ex": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _P, _P, _L, _P],
                          _I),
    "fp4attn_forward": ([_P, _P, _P, _I, _I, _I, _I, _I, _I, _L, _L, _L, _L, _L, _L, _L, _L, _L, _I, _F, _P, _P, _L,
                         _P], _I),
    "fp4attn_forward_ex": ([_P, _P, _P, _I, _I, _I, _I, _I, _I, _L, _L, _L, _L, _L, _L, _L, _L, _L, _I, _F, _I, _P, _P,
                            _L, _P], _I),
    "fp4attn_forward_heads": ([_P, _P, _P, _I, _I, _I, _I, _I, _I, _L, _L, _L, _L, _L, _L, _L, _L, _L, _I, _F, _I, _I,
                               _I, _P, _P, _L, _P], _I),
    "fp4attn_forward_noalloc": ([_P, _P, _P, _I, _I, _I, _I, _I, _I, _L, _L, _L, _L, _L, _L, _L, _L, _L, _I, _F, _P,
                                 _P], _I),
    "nvfp4sim_f32_to_nvf4": ([_P, _P, _P, _L, _P], _I),
    "nvfp4sim_f32_to_nvf4_nosearch": ([_P, _P, _P, _L, _P], _I),
    "nvfp4sim_f16_to_nvf4": ([_P, _P, _P, _L, _P], _I),
    "nvfp4sim_nvf4_to_f32": ([_P, _P, _P, _L, _P], _I),
    "nvfp4sim_nvf4_to_f16": ([_P, _P, _P, _L, _P], _I),
    "fp4q_quantize": ([_P, _I, _I, _I, _I, _I, _L, _L, _L, _I, _I, _I, _F, _P, _L, _P, _I, _L, _P, _P, _I, _L, _P], _I),
    "fp4q_global_scale": ([_P, _I, _I, _I, _I, _I, _L, _L, _L, _I, _I, _F, _P, _P], _I),
}


def load() -> ctypes.CDLL:
    """Load the library (no CUDA needed); raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m fp4_attn_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def call(name: str, *args) -> None:
    """Call an entry point; a non-zero status raises RuntimeError with the library's message."""
    L = load()
    rc = getattr(L, name)(*args)
    if rc != 0:
        msg = L.fp4attn_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed ({rc}): {msg}")


def launch_count() -> int:
    """Kernels launched by libfp4attn.so so far in this process."""
    return int(load().fp4attn_launch_count())


def stream_of(t: torch.Tensor) -> int:
    """The current CUDA stream of t's device, as a raw cudaStream_t."""
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError("fp4_attn_b200 runs on CUDA tensors only (no CPU path)")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()
