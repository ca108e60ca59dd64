"""FP4 attention forward on B200 (host side of csrc/attention.cu).

``fp4_attention_fwd(q, k, v, causal, scaling)`` is the native replacement for
the reference's eager attention with FP4 fake-quant (llama_patch.py:57-105
plus the Q/K/V fake-quant of llama_patch.py:167-196): it takes post-RoPE
query/key/value in the HF layout [B, H, T, D] and returns the attention
output in the layout the reference returns, [B, T, Hq, D], in fp32.

Steps (all on the GPU, no CPU path), one C ABI call (fp4attn_forward_ex):
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
DUAL_Q, DUAL_P, OUT_BF16, PV_FP16 = 1, 2, 4, 8  # fp4attn_forward_ex flags


class AttentionWorkspace:
    """Packed operands of one attention call (reusable across calls of the same shape).

    One device buffer laid out by fp4attn_workspace_layout, with a tensor
    view per piece: qc/kc codes [B*Tp, H*D/2], qs/ks tcgen05 scale atoms,
    gq/gk per-token global scales [B*Tp], vhi/vlo V-hat planes [B*Hkv*D, Tp],
    row_max the row maxima of the scores [B, Hq, Tp] (single-slice Q).
    """

    def __init__(self, B, Hq, Hkv, T, D, device, dual_q: bool = False):
        import ctypes
        self.shape = (B, Hq, Hkv, T, D)
        self.dual_q = bool(dual_q)
        self.flags = DUAL_Q if dual_q else 0
        self.Tp = (T + 127) // 128 * 128
        Tp = self.Tp
        offs = (ctypes.c_int64 * 13)()
        size = _lib.load().fp4attn_workspace_layout_ex(B, Hq, Hkv, T, D, self.flags, offs)
        if size < 0:
            raise ValueError(f"unsupported attention shape B={B} Hq={Hq} Hkv={Hkv} T={T} D={D}")
        self.nbytes = int(size)
        self.buf = torch.empty(self.nbytes + 256, dtype=torch.uint8, device=device)
        base = (-self.buf.data_ptr()) % 256  # 256-byte aligned start
        self.base = base
        o = [int(x) + base for x in offs]
        u8, f32, f16 = torch.uint8, torch.float32, torch.float16

        def view(i, dtype, shape):
            n = 1
            for d in shape:
                n *= d
            esz = torch.empty((), dtype=dtype).element_size()
            return self.buf[o[i]:o[i] + n * esz].view(dtype).view(*shape)

        self.qc = view(0, u8, (B * Tp, Hq * D // 2))
        self.qs = view(1, u8, (B * Tp // 128 * Hq * (D // 64) * 512,))
        self.gq = view(2, f32, (B * Tp,))
        self.kc = view(3, u8, (B * Tp, Hkv * D // 2))
        self.ks = view(4, u8, (B * Tp // 128 * Hkv * (D // 64) * 512,))
        self.gk = view(5, f32, (B * Tp,))
        self.vhi = view(6, f16, (B * Hkv * D, Tp))
        self.vlo = view(7, f16, (B * Hkv * D, Tp))
        if dual_q:  # the residual Q slice (fp4attn_workspace_layout_ex pieces 8-11)
            self.qc_lo = view(8, u8, (B * Tp, Hq * D // 2))
            self.qs_lo = view(9, u8, (B * Tp // 128 * Hq * (D // 64) * 512,))
            self.gq_lo = view(10, f32, (B * Tp,))
            self.row_max = None
        else:  # row maxima of the scores, written by the row-maximum kernel (piece 12)
            self.row_max = view(12, f32, (B, Hq, Tp))

    def ptr(self) -> int:
        return self.buf.data_ptr() + self.base


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
                      workspace: AttentionWorkspace | None = None, num_ctas: int = 0,
                      dual_q: bool = False, dual_p: bool = False,
                      out_dtype: torch.dtype = torch.float32,
                      kv_heads: tuple[int, int] | None = None, pv_fp16: bool = False) -> torch.Tensor:
    """NVFP4 attention forward.  q [B,Hq,T,D], k/v [B,Hkv,T,D] (CUDA) -> [B,T,Hq,D] in out_dtype.

    kv_heads=(h0, h1) attends only KV heads h0..h1-1 and their query groups
    (one rank's shard of a job split by (batch, KV head)) and returns
    [B, T, (h1-h0)*Hq/Hkv, D].  Q/K/V are still quantized on every head of the
    given batch rows, since the reference's per-token global scales span the
    whole [B*T, H*D] row (llama_patch.py:167-196): the attended heads' output
    equals the unsharded call's bit for bit.

    out_dtype fp32 or bf16 (the reference's output dtype for bf16 inputs,
    llama_patch.py:102-103: the kernel rounds its fp32 result once).

    pv_fp16=True (FP4ATTN_PV_FP16) multiplies P-hat by V-hat rounded once to
    fp16 for every query past the first 128 of a sequence, half the PV tensor
    work; the first 128 queries, whose outputs average few keys, keep the exact
    hi + lo planes.  Measured against the exact V-hat: max-abs 2.7e-3 x RMS(O)
    on the Llama-3-8B shape, inside the attention tolerance.

    One call of the C ABI's fp4attn_forward_ex (quantize Q/K, prepare V-hat,
    attention) with the packed operands in ``workspace``.  dual_q / dual_p
    select the reference's dual-slice Q / P (FP4_USE_DUAL_QUANT_Q /
    FP4_USE_DUAL_QUANT_ATTN, llama_patch.py:84,183; dual_nvfp4,
    fp4_quant_utils.py:307-315).
    """
    _lib.require_cuda(q, k, v)
    q, k, v = _bhtd(q), _bhtd(k), _bhtd(v)
    if not (q.dtype == k.dtype == v.dtype):
        dt = torch.float32
        q, k, v = q.to(dt), k.to(dt), v.to(dt)
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    if D != HEAD_DIM:
        raise NotImplementedError(f"head_dim {D}: the tcgen05 kernel implements head_dim {HEAD_DIM}")
    if k.shape != (B, Hkv, T, D) or v.shape != (B, Hkv, T, D) or Hq % Hkv:
        raise ValueError("q [B,Hq,T,D], k/v [B,Hkv,T,D] with Hq % Hkv == 0 expected")
    if scaling is None:
        scaling = D ** -0.5
    ws = workspace or AttentionWorkspace(B, Hq, Hkv, T, D, q.device, dual_q=dual_q)
    if ws.shape != (B, Hq, Hkv, T, D):
        raise ValueError(f"workspace made for {ws.shape}, called with {(B, Hq, Hkv, T, D)}")
    if dual_q and not ws.dual_q:
        raise ValueError("dual_q needs a workspace made with dual_q=True")
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("out_dtype must be torch.float32 or torch.bfloat16")
    if num_ctas and (dual_q or dual_p or out_dtype != torch.float32):
        raise ValueError("num_ctas is a single-slice fp32-output profiling option")
    h0, h1 = (0, Hkv) if kv_heads is None else (int(kv_heads[0]), int(kv_heads[1]))
    if not 0 <= h0 < h1 <= Hkv:
        raise ValueError(f"kv_heads {kv_heads} outside [0, {Hkv})")
    if (h0, h1) != (0, Hkv) and num_ctas:
        raise ValueError("num_ctas is not available with kv_heads")
    Ho = (h1 - h0) * (Hq // Hkv)
    if out is None:
        out = torch.empty(B, T, Ho, D, dtype=out_dtype, device=q.device)
    elif out.shape != (B, T, Ho, D) or out.dtype != out_dtype or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous {out_dtype} [B, T, {Ho}, D] tensor")
    if num_ctas:
        quantize_qk(q, ws.qc, ws.qs, ws.gq, ws.Tp)
        quantize_qk(k, ws.kc, ws.ks, ws.gk, ws.Tp)
        prepare_v(v, ws.vhi, ws.vlo, ws.Tp)
        _lib.call("fp4attn_fwd_packed", ws.qc.data_ptr(), ws.qs.data_ptr(), ws.gq.data_ptr(), ws.kc.data_ptr(),
                  ws.ks.data_ptr(), ws.gk.data_ptr(), ws.vhi.data_ptr(), ws.vlo.data_ptr(), out.data_ptr(), B, Hq,
                  Hkv, T, ws.Tp, D, 1 if causal else 0, float(scaling), int(num_ctas), _lib.stream_of(q))
        return out
    flags = (DUAL_Q if dual_q else 0) | (DUAL_P if dual_p else 0) | \
        (OUT_BF16 if out_dtype == torch.bfloat16 else 0) | (PV_FP16 if pv_fp16 else 0)
    _lib.call("fp4attn_forward_heads", q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.DTYPE_CODE[q.dtype], B, Hq,
              Hkv, T, D, q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2), v.stride(0),
              v.stride(1), v.stride(2), 1 if causal else 0, float(scaling), flags, h0, h1, out.data_ptr(), ws.ptr(),
              ws.nbytes, _lib.stream_of(q))
    return out
