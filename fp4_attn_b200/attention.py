"""FP4 attention forward on B200 (host side of csrc/attention.cu).

``fp4_attention_fwd(q, k, v, causal, scaling)`` is the native replacement for
the reference's eager attention with FP4 fake-quant (llama_patch.py:57-105
plus the Q/K/V fake-quant of llama_patch.py:167-196): it takes post-RoPE
query/key/value in the HF layout [B, H, T, D] and returns the attention
output in the layout the reference returns, [B, T, Hq, D], in fp32.

Steps (all on the GPU, no CPU path):
  1. Q and K -> NVFP4 codes + E4M3 scales (tcgen05 layout) + per-token global
     scale, on their [B*T, H*D] views (fp4q_quantize, row mode);
  2. V -> Vhat (NVFP4 along tokens, per-token global scale) as fp16 hi/lo
     planes (fp4attn_prepare_v);
  3. the tcgen05 attention kernel (fp4attn_fwd_packed).
"""
from __future__ import annotations

import torch

from . import _lib

HEAD_DIM = 128


class AttentionWorkspace:
    """Packed operands of one attention call (reusable across calls of the same shape)."""

    def __init__(self, B, Hq, Hkv, T, D, device):
        self.shape = (B, Hq, Hkv, T, D)
        self.Tp = (T + 127) // 128 * 128
        Tp = self.Tp
        u8 = torch.uint8
        self.qc = torch.empty(B * Tp, Hq * D // 2, dtype=u8, device=device)
        self.qs = torch.empty(B * Tp // 128 * Hq * (D // 64) * 512, dtype=u8, device=device)
        self.gq = torch.empty(B * Tp, dtype=torch.float32, device=device)
        self.kc = torch.empty(B * Tp, Hkv * D // 2, dtype=u8, device=device)
        self.ks = torch.empty(B * Tp // 128 * Hkv * (D // 64) * 512, dtype=u8, device=device)
        self.gk = torch.empty(B * Tp, dtype=torch.float32, device=device)
        self.vhi = torch.empty(B * Hkv * D, Tp, dtype=torch.float16, device=device)
        self.vlo = torch.empty(B * Hkv * D, Tp, dtype=torch.float16, device=device)


def _bhtd(x: torch.Tensor) -> torch.Tensor:
    if x.dtype not in _lib.DTYPE_CODE:
        x = x.float()
    if x.stride(-1) != 1 or x.data_ptr() % 16:
        x = x.contiguous()
    return x


def quantize_qk(x: torch.Tensor, codes, scales, g, Tp: int) -> None:
    """[B,H,T,D] -> NVFP4 operand of the [B*T, H*D] view (row mode, tcgen05 scales)."""
    B, H, T, D = x.shape
    _lib.call("fp4q_quantize", x.data_ptr(), _lib.DTYPE_CODE[x.dtype], B, T, H, D, x.stride(0), x.stride(2),
              x.stride(1), Tp, 1, 0, 1536.0, codes.data_ptr(), codes.shape[1], scales.data_ptr(), 1, H * D // 64,
              g.data_ptr(), None, 0, 0, _lib.stream_of(x))


def prepare_v(v: torch.Tensor, vhi, vlo, Tp: int, vhat=None, g=None) -> None:
    """[B,Hkv,T,D] -> Vhat hi/lo planes [B*Hkv*D, Tp] (optionally fp32 Vhat and the per-token g)."""
    B, H, T, D = v.shape
    _lib.call("fp4attn_prepare_v", v.data_ptr(), _lib.DTYPE_CODE[v.dtype], B, H, T, D, v.stride(0), v.stride(1),
              v.stride(2), Tp, vhi.data_ptr(), vlo.data_ptr(), _lib.ptr(vhat), _lib.ptr(g), _lib.stream_of(v))


def fp4_attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                      scaling: float | None = None, out: torch.Tensor | None = None,
                      workspace: AttentionWorkspace | None = None, num_ctas: int = 0) -> torch.Tensor:
    """NVFP4 attention forward.  q [B,Hq,T,D], k/v [B,Hkv,T,D] (CUDA) -> fp32 [B,T,Hq,D]."""
    _lib.require_cuda(q, k, v)
    q, k, v = _bhtd(q), _bhtd(k), _bhtd(v)
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    if D != HEAD_DIM:
        raise NotImplementedError(f"head_dim {D}: the tcgen05 kernel implements head_dim {HEAD_DIM}")
    if k.shape != (B, Hkv, T, D) or v.shape != (B, Hkv, T, D) or Hq % Hkv:
        raise ValueError("q [B,Hq,T,D], k/v [B,Hkv,T,D] with Hq % Hkv == 0 expected")
    if scaling is None:
        scaling = D ** -0.5
    ws = workspace or AttentionWorkspace(B, Hq, Hkv, T, D, q.device)
    Tp = ws.Tp
    quantize_qk(q, ws.qc, ws.qs, ws.gq, Tp)
    quantize_qk(k, ws.kc, ws.ks, ws.gk, Tp)
    prepare_v(v, ws.vhi, ws.vlo, Tp)
    if out is None:
        out = torch.empty(B, T, Hq, D, dtype=torch.float32, device=q.device)
    _lib.call("fp4attn_fwd_packed", ws.qc.data_ptr(), ws.qs.data_ptr(), ws.gq.data_ptr(), ws.kc.data_ptr(),
              ws.ks.data_ptr(), ws.gk.data_ptr(), ws.vhi.data_ptr(), ws.vlo.data_ptr(), out.data_ptr(), B, Hq, Hkv,
              T, Tp, D, 1 if causal else 0, float(scaling), int(num_ctas), _lib.stream_of(q))
    return out
