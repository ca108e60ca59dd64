"""Python face of the C quantizer oracle (``oracle/nvfp4_oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
bench.py's CPU legs, never by the ``fp4_attn_b200`` package.

Everything here works on numpy arrays.  Two flavours of the reference are
exposed:

* ``fused_qdq`` -- ``FP4Quantizer.single_nvfp4_quant_dequant_fused``
  (fp4_quant_utils.py:112-172): dequantized output plus the codes, E4M3 scale
  bytes and global scales implied by it.
* ``cuda_to_nvf4`` / ``cuda_from_nvf4`` -- the nvfp4sim CUDA kernels
  (fast_fp4/nvfp4sim.cu:96-192, 292-344, 403-499).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")

ARITH = {"float32": 0, "bfloat16": 1, "float16": 2}
GMODE = {"none": 0, "row": 1, "col": 2}

_lib = None


def build() -> str:
    """Compile the C oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        i64 = ctypes.c_int64
        L.oracle_fused_qdq.argtypes = [P, i64, i64, i64, i64, ctypes.c_int, ctypes.c_int, ctypes.c_float, P, P, P, P]
        L.oracle_cuda_f32_to_nvf4.argtypes = [P, P, P, i64, ctypes.c_int]
        L.oracle_cuda_nvf4_to_f32.argtypes = [P, P, P, i64]
        L.oracle_decode_codes.argtypes = [P, P, P, i64, i64]
        L.oracle_e4m3_from_f32_torch.argtypes = [ctypes.c_float]
        L.oracle_e4m3_from_f32_torch.restype = ctypes.c_uint8
        L.oracle_e4m3_from_f32_satfinite.argtypes = [ctypes.c_float]
        L.oracle_e4m3_from_f32_satfinite.restype = ctypes.c_uint8
        L.oracle_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.oracle_e4m3_to_f32.restype = ctypes.c_float
        _lib = L
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def fused_qdq(x: np.ndarray, gmode: str = "row", arith: str = "float32", global_sf_max: float | None = 1536.0):
    """Restatement of single_nvfp4_quant_dequant_fused on a 2-D array.

    ``x`` holds the input tensor's values widened to float32 (any strides).
    ``gmode``: "row" (global_scale_aligned=True), "col" (False) or "none"
    (global_sf_max=None).  Returns (out [m,n], codes [m,npad/2] uint8,
    scales [m,npad/16] uint8, g) with g of shape [m] (row), [npad] (col) or
    None.
    """
    if global_sf_max is None:
        gmode = "none"
    x = np.asarray(x, dtype=np.float32)
    assert x.ndim == 2
    m, n = x.shape
    npad = (n + 15) // 16 * 16
    itemsize = x.itemsize
    out = np.empty((m, n), np.float32)
    codes = np.empty((m, npad // 2), np.uint8)
    scales = np.empty((m, npad // 16), np.uint8)
    g = None
    if gmode == "row":
        g = np.empty((m,), np.float32)
    elif gmode == "col":
        g = np.empty((npad,), np.float32)
    lib().oracle_fused_qdq(_ptr(x), m, n, x.strides[0] // itemsize, x.strides[1] // itemsize,
                           GMODE[gmode], ARITH[arith], float(global_sf_max or 0.0),
                           _ptr(out), _ptr(codes), _ptr(scales), _ptr(g))
    return out, codes, scales, g


def cuda_to_nvf4(x: np.ndarray, search: bool):
    """nvfp4sim.f32_to_nvf4 (search) / f32_to_nvf4_nosearch on [M,16] float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    assert x.ndim == 2 and x.shape[1] == 16
    M = x.shape[0]
    xq = np.zeros((M,), np.uint64)
    xs = np.zeros((M,), np.uint8)
    lib().oracle_cuda_f32_to_nvf4(_ptr(xq), _ptr(xs), _ptr(x), M, int(bool(search)))
    return xq, xs


def cuda_from_nvf4(xq: np.ndarray, xs: np.ndarray) -> np.ndarray:
    """nvfp4sim.nvf4_to_f32: [M] uint64 codes + [M] e4m3 bytes -> [M,16] float32."""
    xq = np.ascontiguousarray(xq, dtype=np.uint64)
    xs = np.ascontiguousarray(xs, dtype=np.uint8)
    M = xq.shape[0]
    out = np.empty((M, 16), np.float32)
    lib().oracle_cuda_nvf4_to_f32(_ptr(out), _ptr(xq), _ptr(xs), M)
    return out


def decode_codes(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """codes [m, npad/2] + scales [m, npad/16] -> q*s as float32 [m, npad]."""
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    m, half = codes.shape
    out = np.empty((m, half * 2), np.float32)
    lib().oracle_decode_codes(_ptr(out), _ptr(codes), _ptr(scales), m, half * 2)
    return out


def e4m3_from_f32_torch(v: float) -> int:
    return int(lib().oracle_e4m3_from_f32_torch(float(v)))


def e4m3_from_f32_satfinite(v: float) -> int:
    return int(lib().oracle_e4m3_from_f32_satfinite(float(v)))


def e4m3_to_f32(b: int) -> float:
    return float(lib().oracle_e4m3_to_f32(int(b)))
