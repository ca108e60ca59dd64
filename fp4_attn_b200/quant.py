"""NVFP4 block-16 quantization on the GPU (host side of csrc/quant.cu).

``quantize`` returns the packed form (E2M1 codes two per byte, E4M3 block
scales, fp32 global scales); ``qdq`` returns the dequantized tensor that
FP4Quantizer.single_nvfp4_quant_dequant_fused (fp4_quant_utils.py:112-172)
returns, bit for bit.

Global-scale modes (``mode``):
  "row"    global_scale_aligned=True: g = rowmax|x| (the reference does not
           divide by global_sf_max on this branch, fp4_quant_utils.py:134,139)
  "col"    global_scale_aligned=False: g = colmax|x| * recip(global_sf_max)
  "none"   global_sf_max=None: no global scale
  "tensor" g = max|x| * recip(global_sf_max), then the row-mode formulas:
           equal to running the reference with global_sf_max=None on
           x * recip(g) and multiplying its output by g
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib

MODES = {"none": 0, "row": 1, "col": 2, "tensor": 3}
SCALE_LAYOUTS = {"linear": 0, "tcgen05": 1}


@dataclass
class NVFP4Tensor:
    """Packed NVFP4 data of a 2-D [m, n] tensor.

    codes  uint8 [m, npad/2]: element 2k in the low nibble of byte k
    scales uint8 (E4M3 bytes): [m, npad/16] ("linear") or tcgen05 atoms
    g      float32 global scale: [m] (row), [npad] (col), [1] (tensor), None
    """
    codes: torch.Tensor
    scales: torch.Tensor
    g: torch.Tensor | None
    shape: tuple
    mode: str
    scale_layout: str

    def scales_e4m3(self) -> torch.Tensor:
        return self.scales.view(torch.float8_e4m3fn)


def _prep(x: torch.Tensor, dequant_dtype: torch.dtype) -> torch.Tensor:
    _lib.require_cuda(x)
    if x.dim() != 2:
        raise ValueError("expected a 2-D tensor")
    if x.dtype not in _lib.DTYPE_CODE:
        x = x.to(dequant_dtype)
    if x.stride(1) != 1:
        x = x.contiguous()
    return x


def _run(x, mode, global_sf_max, dequant_dtype, codes, scales, scale_layout, scales_ld, g, out, out_ld):
    m, n = x.shape
    if mode not in MODES:
        raise ValueError(f"mode must be one of {list(MODES)}")
    if dequant_dtype not in _lib.DTYPE_CODE:
        raise ValueError("dequant_dtype must be float32, bfloat16 or float16")
    _lib.call("fp4q_quantize", x.data_ptr(), _lib.DTYPE_CODE[x.dtype], 1, m, 1, n, 0, x.stride(0), 0, m,
              MODES[mode], _lib.DTYPE_CODE[dequant_dtype], float(global_sf_max or 0.0),
              _lib.ptr(codes), codes.shape[1] if codes is not None else 0,
              _lib.ptr(scales), SCALE_LAYOUTS[scale_layout], scales_ld,
              _lib.ptr(g), _lib.ptr(out), _lib.DTYPE_CODE[out.dtype] if out is not None else 0, out_ld,
              _lib.stream_of(x))


def _g_buffer(mode, m, npad, device):
    if mode == "row":
        return torch.empty(m, dtype=torch.float32, device=device)
    if mode == "col":
        return torch.empty(npad, dtype=torch.float32, device=device)
    if mode == "tensor":
        return torch.empty(1, dtype=torch.float32, device=device)
    return None


def quantize(x: torch.Tensor, mode: str = "row", global_sf_max: float | None = 1536.0,
             dequant_dtype: torch.dtype = torch.float32, scale_layout: str = "linear") -> NVFP4Tensor:
    """Quantize a 2-D CUDA tensor to packed NVFP4 (block 16 along the last dim)."""
    if global_sf_max is None:
        mode = "none"
    x = _prep(x, dequant_dtype)
    m, n = x.shape
    npad = (n + 15) // 16 * 16
    nblk = npad // 16
    codes = torch.empty(m, npad // 2, dtype=torch.uint8, device=x.device)
    if scale_layout == "tcgen05":
        nkb4 = (nblk + 3) // 4
        mpad = (m + 127) // 128 * 128
        scales = torch.zeros(mpad * nkb4 * 4, dtype=torch.uint8, device=x.device)
        scales_ld = nkb4
    else:
        scales = torch.empty(m, nblk, dtype=torch.uint8, device=x.device)
        scales_ld = nblk
    g = _g_buffer(mode, m, npad, x.device)
    if m:
        _run(x, mode, global_sf_max, dequant_dtype, codes, scales, scale_layout, scales_ld, g, None, 0)
    return NVFP4Tensor(codes, scales, g, (m, n), mode, scale_layout)


def qdq(x: torch.Tensor, mode: str = "row", global_sf_max: float | None = 1536.0,
        dequant_dtype: torch.dtype = torch.float32, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Fused quantize -> dequantize; returns [m, n] in ``out_dtype`` (default: the dequant dtype)."""
    if global_sf_max is None:
        mode = "none"
    x = _prep(x, dequant_dtype)
    m, n = x.shape
    npad = (n + 15) // 16 * 16
    out = torch.empty(m, n, dtype=out_dtype or dequant_dtype, device=x.device)
    g = _g_buffer(mode, m, npad, x.device)
    if m and n:
        _run(x, mode, global_sf_max, dequant_dtype, None, None, "linear", 0, g, out, n)
    return out


def dequantize(t: NVFP4Tensor, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """codes * scale * g back to [m, n] (fp32 arithmetic, one rounding to out_dtype)."""
    m, n = t.shape
    lo = (t.codes & 15).to(torch.int64)
    hi = (t.codes >> 4).to(torch.int64)
    nib = torch.stack((lo, hi), dim=-1).reshape(m, -1)
    grid = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], device=t.codes.device)
    val = grid[nib & 7] * torch.where((nib & 8) != 0, -1.0, 1.0)
    if t.scale_layout != "linear":
        raise ValueError("dequantize expects the linear scale layout")
    s = t.scales_e4m3().float().repeat_interleave(16, dim=1)
    y = val * s
    if t.mode in ("row",):
        y = y * t.g[:, None]
    elif t.mode == "col":
        y = y * t.g[None, :]
    elif t.mode == "tensor":
        y = y * t.g
    return y[:, :n].to(out_dtype)
