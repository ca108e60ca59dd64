"""fp4_attn_b200: the NVFP4 quantizer and FP4 attention forward of
tg-together/fp4_attn, rebuilt as hand-written sm_100a CUDA kernels behind the
reference's own Python API.

* ``fp4_attn_b200.fp4_quant_utils.FP4Quantizer`` -- drop-in for the
  reference's FP4Quantizer (fp4_quant_utils.py).
* ``fp4_attn_b200.nvfp4sim``  -- drop-in for the reference's CUDA extension
  module of the same name (fast_fp4/).
* ``fp4_attn_b200.quant``     -- packed NVFP4 quantize / dequantize.

The compute path is libfp4attn.so (C ABI in include/fp4attn.h), built
in-tree by ``python -m fp4_attn_b200.build``.
"""
from . import quant  # noqa: F401
from .fp4_quant_utils import FP4Quantizer  # noqa: F401

__all__ = ["FP4Quantizer", "quant"]
