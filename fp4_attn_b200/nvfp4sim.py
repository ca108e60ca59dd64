"""Drop-in for the reference extension module ``nvfp4sim``.

Same five functions, argument order and tensor conventions as the pybind11
module built from fast_fp4/wrapper.cpp:40-46 (host code
fast_fp4/nvfp4sim.cu:156-499): caller-allocated outputs first, ``M`` groups
of 16, ``M`` even, work enqueued on the current CUDA stream.  Misuse raises
``RuntimeError`` where the reference either raised (TORCH_CHECK) or aborted
the process (C ``assert``).

``import fp4_attn_b200.nvfp4sim as nvfp4sim`` (or register it in
``sys.modules["nvfp4sim"]``) lets fp4_quant_utils.py:13 run unchanged.
"""
from __future__ import annotations

import torch

from . import _lib


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_io(q: torch.Tensor, s: torch.Tensor, x: torch.Tensor, x_dtype: torch.dtype, x_name: str) -> int:
    for t, n in ((q, "XQ"), (s, "XS"), (x, x_name)):
        _check(t.is_cuda, f"{n} must be a CUDA tensor")
        _check(t.is_contiguous(), f"{n} must be contiguous")
    _check(q.dim() == 1 and s.dim() == 1, "codes and scales must be 1-D")
    _check(x.dim() == 2 and x.shape[1] == 16, f"{x_name} must be [M, 16]")
    M = x.shape[0]
    _check(q.shape[0] == M and s.shape[0] == M, "codes/scales length must equal M")
    _check(M % 2 == 0, "M must be even")
    _check(q.dtype == torch.int64, "codes must be int64")
    _check(s.dtype == torch.float8_e4m3fn, "scales must be float8_e4m3fn")
    _check(x.dtype == x_dtype, f"{x_name} must be {x_dtype}")
    _check(q.device == s.device == x.device, "tensors must share a device")
    return M


def f32_to_nvf4(XQout: torch.Tensor, XSout: torch.Tensor, Xin: torch.Tensor) -> None:
    """float32 [M,16] -> codes int64[M] + E4M3 scales, 16-candidate scale search."""
    M = _check_io(XQout, XSout, Xin, torch.float32, "Xin")
    _lib.call("nvfp4sim_f32_to_nvf4", XQout.data_ptr(), XSout.data_ptr(), Xin.data_ptr(), M, _lib.stream_of(Xin))


def f32_to_nvf4_nosearch(XQout: torch.Tensor, XSout: torch.Tensor, Xin: torch.Tensor) -> None:
    """float32 [M,16] -> codes + scales with the amax/6 scale only."""
    M = _check_io(XQout, XSout, Xin, torch.float32, "Xin")
    _lib.call("nvfp4sim_f32_to_nvf4_nosearch", XQout.data_ptr(), XSout.data_ptr(), Xin.data_ptr(), M,
              _lib.stream_of(Xin))


def f16_to_nvf4(XQout: torch.Tensor, XSout: torch.Tensor, Xin: torch.Tensor) -> None:
    """float16 [M,16] -> codes + scales, 16-candidate scale search."""
    M = _check_io(XQout, XSout, Xin, torch.float16, "Xin")
    _lib.call("nvfp4sim_f16_to_nvf4", XQout.data_ptr(), XSout.data_ptr(), Xin.data_ptr(), M, _lib.stream_of(Xin))


def nvf4_to_f32(Xout: torch.Tensor, XQin: torch.Tensor, XSin: torch.Tensor) -> None:
    """codes + scales -> float32 [M,16]."""
    M = _check_io(XQin, XSin, Xout, torch.float32, "Xout")
    _lib.call("nvfp4sim_nvf4_to_f32", Xout.data_ptr(), XQin.data_ptr(), XSin.data_ptr(), M, _lib.stream_of(Xout))


def nvf4_to_f16(Xout: torch.Tensor, XQin: torch.Tensor, XSin: torch.Tensor) -> None:
    """codes + scales -> float16 [M,16]."""
    M = _check_io(XQin, XSin, Xout, torch.float16, "Xout")
    _lib.call("nvfp4sim_nvf4_to_f16", Xout.data_ptr(), XQin.data_ptr(), XSin.data_ptr(), M, _lib.stream_of(Xout))


# ---------------------------------------------------------------------------
# Exports added next to the five reference functions: the packed quantizer,
# its inverse, the fused round trip and the FP4 attention forward.  They have
# no counterpart in the reference's extension (wrapper.cpp:40-46); they are
# the calls its Python layer makes through torch ops today
# (fp4_quant_utils.py:112-172, llama_patch.py:57-105 and 167-196).

def quantize_nvfp4(x: torch.Tensor, mode: str = "row", global_sf_max: float | None = 1536.0, search: bool = False,
                   scale_layout: str = "linear", dequant_dtype: torch.dtype = torch.float32):
    """x [m, n] (CUDA) -> (codes uint8 [m, npad/2], scales E4M3 bytes, g fp32 or None)."""
    from . import quant
    if search:
        raise NotImplementedError("the scale search packs through f32_to_nvf4 ([M,16] groups), not quantize_nvfp4")
    t = quant.quantize(x, mode, global_sf_max, dequant_dtype, scale_layout)
    return t.codes, t.scales, t.g


def dequantize_nvfp4(codes: torch.Tensor, scales: torch.Tensor, g: torch.Tensor | None, shape, mode: str = "row",
                     out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Inverse of quantize_nvfp4 (linear scale layout): code * scale * g."""
    from . import quant
    t = quant.NVFP4Tensor(codes, scales, g, tuple(shape), mode if g is not None else "none", "linear")
    return quant.dequantize(t, out_dtype)


def qdq_nvfp4(x: torch.Tensor, mode: str = "row", global_sf_max: float | None = 1536.0,
              dequant_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """single_nvfp4_quant_dequant_fused (fp4_quant_utils.py:112-172) on the GPU, bit for bit."""
    from . import quant
    return quant.qdq(x, mode, global_sf_max, dequant_dtype)


def fp4_attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                      scaling: float | None = None, dual_q: bool = False, dual_p: bool = False,
                      v_scale_mode: str = "token") -> torch.Tensor:
    """Q/K/V fake-quant + FP4 attention (llama_patch.py:57-105, 167-196): [B,Hq,T,D] -> fp32 [B,T,Hq,D].

    dual_q / dual_p: the reference's residual two-slice quantization of Q / P
    (dual_nvfp4, fp4_quant_utils.py:307-315).  V scales other than per token
    (the reference's global_scale_aligned=False) are not implemented and raise.
    """
    from .attention import fp4_attention_fwd as fwd
    if v_scale_mode != "token":
        raise NotImplementedError("V is quantized along tokens with a per-token global scale only")
    return fwd(q, k, v, causal=causal, scaling=scaling, dual_q=dual_q, dual_p=dual_p)
