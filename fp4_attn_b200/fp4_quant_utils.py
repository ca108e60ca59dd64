"""Drop-in ``FP4Quantizer`` backed by the sm_100a kernels.

Mirrors fp4_quant_utils.py:17-341 of the reference: same constructor
arguments, attributes and methods, same results (bit-exact on the torch path,
bit-exact to the reference CUDA extension on the search path).  Differences,
all outside the numbers:

* inputs must be CUDA tensors (the kernels are the only compute path);
* ``single_nvfp4_quant_dequant_fused`` no longer prints or empties the CUDA
  cache on every call (fp4_quant_utils.py:115,117,171);
* ``single_nvfp4_qd_nosearch`` / ``single_nvfp4_qd_searched`` work for
  every shape (the reference raises UnboundLocalError when no padding is
  needed, :204-223);
* ``single_nvfp4_fake_quant`` / ``dual_nvfp4_fake_quant``, which
  llama_patch.py:94,96,189-196 calls but the reference only has as comments
  (:322-335), are provided: the single/dual result cast to the input dtype.
"""
from __future__ import annotations

import torch
from torch import Tensor, nn

from . import nvfp4sim, quant


class FP4Quantizer(nn.Module):
    """FP4 quantizer: NVFP4 (E2M1 values, E4M3 scale per 16, fp32 global scale) fake-quant."""

    def __init__(self, block_size: int = 16, float4_e2m1_max: float = 6.0, float8_e4m3_max: float = 448.0,
                 global_sf_max=256 * 6, dequant_dtype: torch.dtype = torch.float32):
        super().__init__()
        if block_size != 16 or float4_e2m1_max != 6.0 or float8_e4m3_max != 448.0:
            raise NotImplementedError("the NVFP4 kernels implement block 16, E2M1 max 6, E4M3 max 448")
        self.block_size = block_size
        self.float4_e2m1_max = torch.tensor(float4_e2m1_max, dtype=dequant_dtype)
        self.float8_e4m3_max = torch.tensor(float8_e4m3_max, dtype=dequant_dtype)
        self.global_sf_max = None if global_sf_max is None else torch.tensor(global_sf_max, dtype=dequant_dtype)
        self.zero_tensor = torch.tensor(0.0, dtype=dequant_dtype)
        self.one_tensor = torch.tensor(1.0, dtype=dequant_dtype)
        self.dequant_dtype = dequant_dtype

    # --- elementwise helpers (fp4_quant_utils.py:47-69) -------------------
    def cast_to_fp4(self, x: Tensor) -> Tensor:
        """Round to the E2M1 grid, ties to even, sign from torch.sign."""
        a = torch.abs(x)
        step = torch.where(a < 2, 0.5, torch.where(a < 4, 1.0, 2.0)).to(x.dtype)
        q = torch.where(a > 6, torch.full_like(a, 6.0), torch.round(a / step) * step)
        return q * torch.sign(x)

    def get_reciprocal(self, x):
        if isinstance(x, torch.Tensor):
            one = self.one_tensor.to(x.device)
            return torch.where(x == 0, 0.0, one / x)
        raise TypeError("Input must be a torch.Tensor.")

    def _gsf(self) -> float | None:
        return None if self.global_sf_max is None else float(self.global_sf_max)

    # --- torch path (fp4_quant_utils.py:112-172) ---------------------------
    def single_nvfp4_quant_dequant_fused(self, x: Tensor, global_scale_aligned: bool = True) -> Tensor:
        if x.dim() != 2:
            raise ValueError("expected a 2-D tensor")
        mode = "row" if global_scale_aligned else "col"
        return quant.qdq(x, mode, self._gsf(), self.dequant_dtype)

    # --- reference CUDA-extension paths (fp4_quant_utils.py:198-305) -------
    def _qd_ext(self, x: Tensor, global_scale_aligned: bool, search: bool) -> Tensor:
        if self.global_sf_max is None:
            raise TypeError("the extension paths need global_sf_max")
        x = x.to(torch.float32)
        m_orig, n_orig = x.shape
        pad_cols = (self.block_size - n_orig % self.block_size) % self.block_size
        pad_rows = m_orig % 2
        if pad_cols or pad_rows:
            x = torch.nn.functional.pad(x, (0, pad_cols, 0, pad_rows), value=0.0)
        m, n = x.shape
        x = x.contiguous()
        dim = 1 if global_scale_aligned else 0
        global_sf = torch.max(abs(x), dim=dim, keepdim=True)[0].to(self.dequant_dtype)
        global_sf = global_sf * self.get_reciprocal(self.global_sf_max.to(x.device))
        x = x * self.get_reciprocal(global_sf)
        x = x.view(m * (n // self.block_size), self.block_size)
        M = x.shape[0]
        q = torch.empty(M, dtype=torch.int64, device=x.device)
        s = torch.empty(M, dtype=torch.float8_e4m3fn, device=x.device)
        (nvfp4sim.f32_to_nvf4 if search else nvfp4sim.f32_to_nvf4_nosearch)(q, s, x)
        rec = torch.empty(M, self.block_size, dtype=torch.float32, device=x.device)
        nvfp4sim.nvf4_to_f32(rec, q, s)
        rec = rec.view(m, n) * global_sf
        return rec[:m_orig, :n_orig].to(torch.bfloat16)

    def single_nvfp4_qd_nosearch(self, x: Tensor, global_scale_aligned: bool = True) -> Tensor:
        return self._qd_ext(x, global_scale_aligned, search=False)

    def single_nvfp4_qd_searched(self, x: Tensor, global_scale_aligned: bool = True) -> Tensor:
        return self._qd_ext(x, global_scale_aligned, search=True)

    # --- dispatch (fp4_quant_utils.py:307-341) -----------------------------
    def dual_nvfp4(self, x: Tensor, global_scale_aligned: bool = True, search: bool = False) -> Tensor:
        """x ~ hi + lo with both slices NVFP4 (residual quantization)."""
        hi = self.single_nvfp4(x, global_scale_aligned, search)
        return hi + self.single_nvfp4(x - hi, global_scale_aligned, search)

    def single_nvfp4(self, x: Tensor, global_scale_aligned: bool = True, search: bool = False) -> Tensor:
        if not search:
            return self.single_nvfp4_quant_dequant_fused(x, global_scale_aligned)
        return self.single_nvfp4_qd_searched(x, global_scale_aligned)

    # --- names llama_patch.py calls (absent from the reference class) ------
    def single_nvfp4_fake_quant(self, x: Tensor, global_scale_aligned: bool = True, search: bool = False) -> Tensor:
        return self.single_nvfp4(x, global_scale_aligned, search).to(x.dtype)

    def dual_nvfp4_fake_quant(self, x: Tensor, global_scale_aligned: bool = True, search: bool = False) -> Tensor:
        return self.dual_nvfp4(x, global_scale_aligned, search).to(x.dtype)

    # --- packed form (new) ---------------------------------------------------
    def quantize(self, x: Tensor, global_scale_aligned: bool = True, scale_layout: str = "linear") -> quant.NVFP4Tensor:
        """Codes + E4M3 scales + global scales of what single_nvfp4_quant_dequant_fused computes."""
        mode = "row" if global_scale_aligned else "col"
        return quant.quantize(x, mode, self._gsf(), self.dequant_dtype, scale_layout)
