"""NVFP4 GEMM on tcgen05 (host side of csrc/gemm_nvf4.cu)."""
from __future__ import annotations

import torch

from . import _lib
from .quant import NVFP4Tensor


def gemm_nvf4(a: NVFP4Tensor, b: NVFP4Tensor) -> torch.Tensor:
    """C = A @ B^T for NVFP4 operands quantized along K with scale_layout="tcgen05".

    Global scales of A (per row, or per tensor) and of B (per row) are applied
    in the epilogue; returns fp32 [M, N].
    """
    if a.scale_layout != "tcgen05" or b.scale_layout != "tcgen05":
        raise ValueError("operands need scale_layout='tcgen05'")
    if a.mode == "col" or b.mode == "col":
        raise ValueError("column global scales vary along K and cannot be factored out of the product")
    M, K = a.shape
    N, K2 = b.shape
    if K != K2:
        raise ValueError("K mismatch")
    dev = a.codes.device
    c = torch.empty(M, N, dtype=torch.float32, device=dev)

    def g(t, rows):
        if t.g is None:
            return None
        return t.g if t.g.numel() == rows else t.g.expand(rows).contiguous()

    ga, gb = g(a, M), g(b, N)
    _lib.call("fp4_gemm_nvf4", a.codes.data_ptr(), a.scales.data_ptr(), _lib.ptr(ga), b.codes.data_ptr(),
              b.scales.data_ptr(), _lib.ptr(gb), c.data_ptr(), M, N, K, a.codes.stride(0), b.codes.stride(0),
              c.stride(0), _lib.stream_of(c))
    return c


def device_status(reset: bool = True) -> int:
    """Non-zero if a bounded wait inside a kernel gave up (synchronizes)."""
    return int(_lib.load().fp4attn_device_status(1 if reset else 0))
