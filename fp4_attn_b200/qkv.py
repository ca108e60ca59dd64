"""Q/K projections fused with RoPE and the NVFP4 row quantizer (host side of csrc/qkv_quant.cu).

The reference's patched attention projects the hidden states (q_proj /
k_proj, llama_patch.py:147-149), fake-quantizes the [B*T, H*D] views
row-wise under a per-token global scale (llama_patch.py:167-194) and rotates
them (llama_patch.py:210).  ``rope_quant_projection`` does the projection,
the rotation (HF apply_rotary_pos_emb in bf16, op for op) and the
quantization of the rotated values in one launch, writing the packed operand
the attention kernel reads; no bf16 Q or K tensor goes to HBM.

``attention_from_hidden`` is the whole attention of one layer from the
hidden states: Q and K through the fused kernel, V through the layer's bf16
linear and fp4attn_prepare_v, then the attention kernel.
"""
from __future__ import annotations

import torch

from . import _lib
from .attention import AttentionWorkspace, OUT_BF16, DUAL_P, prepare_v

HEAD_DIM = 128


def _check_bf16(name: str, t: torch.Tensor, shape: tuple) -> None:
    if t.dtype != torch.bfloat16 or tuple(t.shape) != shape or not t.is_contiguous() or t.data_ptr() % 16:
        raise ValueError(f"{name} must be a contiguous, 16-byte aligned bf16 tensor of shape {shape}")


def rope_quant_projection(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, T: int,
                          codes: torch.Tensor | None = None, scales: torch.Tensor | None = None,
                          g: torch.Tensor | None = None):
    """x [M, K] bf16 hidden states (M = B*T), weight [H*128, K] bf16, cos/sin [M, 128] bf16 per token
    -> (codes uint8 [M, H*64], scales uint8 tcgen05 atoms [M/128 * H*2 * 512], g fp32 [M])."""
    _lib.require_cuda(x, weight, cos, sin)
    M, K = x.shape
    N = weight.shape[0]
    if N % HEAD_DIM:
        raise ValueError("weight rows must be whole heads of 128")
    H = N // HEAD_DIM
    _check_bf16("x", x, (M, K))
    _check_bf16("weight", weight, (N, K))
    _check_bf16("cos", cos, (M, HEAD_DIM))
    _check_bf16("sin", sin, (M, HEAD_DIM))
    dev = x.device
    if codes is None:
        codes = torch.empty(M, N // 2, dtype=torch.uint8, device=dev)
    if scales is None:
        scales = torch.empty(M // 128 * H * 2 * 512, dtype=torch.uint8, device=dev)
    if g is None:
        g = torch.empty(M, dtype=torch.float32, device=dev)
    _lib.call("fp4qkv_rope_quant", x.data_ptr(), weight.data_ptr(), cos.data_ptr(), sin.data_ptr(), M, K, H, T,
              codes.data_ptr(), scales.data_ptr(), g.data_ptr(), _lib.stream_of(x))
    return codes, scales, g


def attention_from_hidden(hidden: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor,
                          cos: torch.Tensor, sin: torch.Tensor, causal: bool = True, scaling: float | None = None,
                          dual_p: bool = False, out_dtype: torch.dtype = torch.bfloat16,
                          workspace: AttentionWorkspace | None = None) -> torch.Tensor:
    """One layer's FP4 attention from hidden [B, T, hidden] bf16 (weights [H*128, hidden] bf16,
    cos/sin [B, T, 128] bf16) -> [B, T, Hq, 128] in out_dtype.  Single-slice Q; T % 128 == 0."""
    _lib.require_cuda(hidden, wq, wk, wv, cos, sin)
    B, T, Kh = hidden.shape
    Hq, Hkv, D = wq.shape[0] // HEAD_DIM, wk.shape[0] // HEAD_DIM, HEAD_DIM
    if T % 128:
        raise NotImplementedError("the fused projection needs T % 128 == 0")
    if scaling is None:
        scaling = D ** -0.5
    ws = workspace or AttentionWorkspace(B, Hq, Hkv, T, D, hidden.device)
    x = hidden.reshape(B * T, Kh)
    c2, s2 = cos.reshape(B * T, D), sin.reshape(B * T, D)
    rope_quant_projection(x, wq, c2, s2, T, ws.qc, ws.qs, ws.gq)
    rope_quant_projection(x, wk, c2, s2, T, ws.kc, ws.ks, ws.gk)
    v = torch.nn.functional.linear(hidden, wv).view(B, T, Hkv, D).transpose(1, 2)  # [B, Hkv, T, D] view
    prepare_v(v, ws.vhi, ws.vlo, ws.Tp)
    out = torch.empty(B, T, Hq, D, dtype=out_dtype, device=hidden.device)
    flags = (OUT_BF16 if out_dtype == torch.bfloat16 else 0) | (DUAL_P if dual_p else 0)
    _lib.call("fp4attn_fwd_packed_dual", ws.qc.data_ptr(), ws.qs.data_ptr(), ws.gq.data_ptr(), None, None, None,
              ws.kc.data_ptr(), ws.ks.data_ptr(), ws.gk.data_ptr(), ws.vhi.data_ptr(), ws.vlo.data_ptr(),
              out.data_ptr(), B, Hq, Hkv, T, ws.Tp, D, 1 if causal else 0, float(scaling), flags, 0,
              _lib.stream_of(hidden))
    return out
