"""Torch (CPU) restatement of the reference quantizer and simulated-FP4 attention.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA attention kernel and the
CPU baseline that bench.py times; never imported by ``fp4_attn_b200``.

``fused_qdq`` follows FP4Quantizer.single_nvfp4_quant_dequant_fused
(fp4_quant_utils.py:112-172) op for op in the dequant dtype, so it is
bit-identical to the reference (checked against tests/golden and against the
C oracle).  The E2M1 rounding is written as round-half-even on a grid whose
step doubles per octave (0.5 below 2, 1 below 4, 2 above); that equals the
reference's eight-threshold cast_to_fp4 (:47-62) on [0, 6].

``attention`` follows llama_patch.py:57-105 (eager_attention_forward with the
P fake-quant on) after the Q/K/V fake-quant of llama_patch.py:167-196, in fp32
simulation precision (the FP4Quantizer default dequant dtype).
"""
from __future__ import annotations

import torch


def _recip(v: torch.Tensor) -> torch.Tensor:
    """get_reciprocal (fp4_quant_utils.py:64-69)."""
    one = torch.ones((), dtype=v.dtype)
    return torch.where(v == 0, torch.zeros((), dtype=v.dtype), one / v)


def e2m1_round(x: torch.Tensor) -> torch.Tensor:
    """cast_to_fp4 (fp4_quant_utils.py:47-62): sign(x) * RNE_E2M1(|x|), x in [-6, 6] or NaN."""
    a = x.abs()
    step = torch.where(a < 2, 0.5, torch.where(a < 4, 1.0, 2.0)).to(x.dtype)
    q = torch.round(a / step) * step
    return q * torch.sign(x)


def fused_qdq(x: torch.Tensor, aligned: bool = True, global_sf_max=1536.0,
              dequant_dtype: torch.dtype = torch.float32, block: int = 16) -> torch.Tensor:
    """single_nvfp4_quant_dequant_fused (fp4_quant_utils.py:112-172)."""
    dt = dequant_dtype
    x = x.to(dt)
    m, n = x.shape
    n_orig = n
    if n % block:
        x = torch.nn.functional.pad(x, (0, block - n % block), value=0.0)
        n = x.shape[1]
    g = None
    if global_sf_max is not None:
        if aligned:
            g = x.abs().amax(dim=1, keepdim=True)  # no division by global_sf_max (:134, :139)
        else:
            gmax = torch.tensor(global_sf_max, dtype=dt)
            g = x.abs().amax(dim=0, keepdim=True) * _recip(gmax)
        x = x * _recip(g)
    x = x.reshape(m, n // block, block)
    s = x.abs().amax(dim=-1, keepdim=True) * _recip(torch.tensor(6.0, dtype=dt))
    s = s.to(torch.float8_e4m3fn).to(dt)
    x = x * _recip(s)
    x = torch.clamp(x, -6.0, 6.0)
    x = e2m1_round(x) * s
    x = x.view(m, n)
    if g is not None:
        x = x * g
    return x[:, :n_orig]


def dual_qdq(x: torch.Tensor, aligned: bool = True, **kw) -> torch.Tensor:
    """dual_nvfp4 without search (fp4_quant_utils.py:313-315)."""
    hi = fused_qdq(x, aligned, **kw)
    return hi + fused_qdq(x - hi, aligned, **kw)


def fake_quant_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, dual_q: bool = False):
    """Q/K/V fake-quant of llama_patch.py:167-208 on [B,H,T,D] tensors (fp32 out).

    Q and K are quantized on their [B*T, H*D] views with a per-token global
    scale; V's view is transposed so blocks run along tokens with a per-token
    global scale (global_scale_aligned=False).
    """
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    q2 = q.permute(0, 2, 1, 3).reshape(B * T, Hq * D).float()
    k2 = k.permute(0, 2, 1, 3).reshape(B * T, Hkv * D).float()
    v2 = v.permute(0, 2, 1, 3).reshape(B * T, Hkv * D).float()
    q2 = dual_qdq(q2) if dual_q else fused_qdq(q2)
    k2 = fused_qdq(k2)
    v2 = fused_qdq(v2.T, aligned=False).T
    Qf = q2.reshape(B, T, Hq, D).permute(0, 2, 1, 3)
    Kf = k2.reshape(B, T, Hkv, D).permute(0, 2, 1, 3)
    Vf = v2.reshape(B, T, Hkv, D).permute(0, 2, 1, 3)
    return Qf, Kf, Vf


def eager_attention(Qf, Kf, Vf, causal: bool, scaling: float, dual_p: bool = False,
                    q_rows: slice | None = None) -> torch.Tensor:
    """eager_attention_forward with P fake-quant (llama_patch.py:57-105), fp32.

    Processes one kv-head group at a time (P quantization is per row, so this
    equals the reference's full-tensor pass).  ``q_rows`` restricts the query
    rows computed (used to time a bounded sample).  Returns [B, Tq, Hq, D].
    """
    B, Hq, T, D = Qf.shape
    Hkv = Kf.shape[1]
    G = Hq // Hkv
    rows = q_rows or slice(0, T)
    r0 = rows.start or 0
    r1 = rows.stop if rows.stop is not None else T
    out = torch.empty(B, r1 - r0, Hq, D, dtype=torch.float32)
    S_len = Kf.shape[2]
    mask = None
    if causal:
        i = torch.arange(r0, r1)[:, None]
        j = torch.arange(S_len)[None, :]
        mask = torch.where(j > i, float("-inf"), 0.0)
    for b in range(B):
        for h in range(Hkv):
            q = Qf[b, h * G:(h + 1) * G, r0:r1]  # [G, Tq, D]
            s = torch.matmul(q, Kf[b, h].transpose(0, 1)) * scaling
            if mask is not None:
                s = s + mask
            p = torch.softmax(s, dim=-1, dtype=torch.float32)
            p2 = p.reshape(-1, S_len)
            p2 = dual_qdq(p2) if dual_p else fused_qdq(p2)
            o = torch.matmul(p2.view(p.shape), Vf[b, h])
            out[b, :, h * G:(h + 1) * G] = o.transpose(0, 1)
    return out


def attention(q, k, v, causal: bool = True, scaling: float | None = None,
              dual_q: bool = False, dual_p: bool = False, q_rows: slice | None = None) -> torch.Tensor:
    """Simulated-FP4 attention from bf16 [B,H,T,D] inputs to fp32 [B,T,Hq,D]."""
    if scaling is None:
        scaling = q.shape[-1] ** -0.5
    Qf, Kf, Vf = fake_quant_qkv(q, k, v, dual_q)
    return eager_attention(Qf, Kf, Vf, causal, scaling, dual_p, q_rows)


# --------------------------------------------------------------------------
# Decision margins of the P quantization.
#
# P's NVFP4 codes are a discontinuous function of S: two correct
# implementations whose S differ in the last bits of fp32 (summation order,
# exp implementation) can round a P element -- or a whole block's E4M3 scale
# -- to neighbouring values, which moves that output row by far more than
# the rounding noise.  The reference itself shows this: recomputing its S in
# float64 instead of fp32 moves a few rows of O by up to ~0.05 x RMS(O).
# ambiguous_rows() flags the rows where any quantization decision of P lies
# within a relative `delta` of a rounding boundary, so a max-abs check can be
# restricted to rows whose FP4 decisions are determined at fp32 precision.

_E2M1_THRESH = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)


def _e4m3_margin(v: torch.Tensor) -> torch.Tensor:
    """Relative distance of v (>= 0) to the nearest E4M3 round-to-nearest boundary."""
    v = v.double()
    e = torch.floor(torch.log2(torch.clamp(v, min=1e-300))).clamp(min=-6)
    step = torch.exp2(e - 3)
    f = v / step
    d = (f - torch.floor(f) - 0.5).abs() * step / torch.clamp(v, min=1e-300)
    return torch.where(v > 0, d, torch.full_like(d, float("inf")))


def ambiguous_rows(S: torch.Tensor, delta: float) -> torch.Tensor:
    """S: scaled, masked scores [..., keys] (float64 preferred).  Returns bool [...]."""
    S = S.double()
    m = S.amax(-1, keepdim=True)
    x = torch.exp(S - m)
    n = x.shape[-1]
    if n % 16:
        x = torch.nn.functional.pad(x, (0, 16 - n % 16))
    xb = x.reshape(*x.shape[:-1], -1, 16)
    sc = xb.amax(-1) * (1.0 / 6.0)
    amb = (_e4m3_margin(sc) < delta).any(-1)
    s = sc.float().to(torch.float8_e4m3fn).double()
    rs = torch.where(s == 0, torch.zeros_like(s), 1.0 / s)
    y = xb * rs[..., None]
    for t in _E2M1_THRESH:
        amb |= ((y - t).abs() / t < delta).flatten(-2).any(-1)
    return amb


def attention_with_margins(q, k, v, causal: bool = True, scaling: float | None = None, delta: float = 1e-5):
    """attention() plus, per output row [B, T, Hq], whether its P quantization is ambiguous at `delta`."""
    if scaling is None:
        scaling = q.shape[-1] ** -0.5
    Qf, Kf, Vf = fake_quant_qkv(q, k, v)
    out = eager_attention(Qf, Kf, Vf, causal, scaling)
    B, Hq, T, D = Qf.shape
    G = Hq // Kf.shape[1]
    flags = torch.zeros(B, T, Hq, dtype=torch.bool)
    mask = torch.triu(torch.full((T, T), float("-inf"), dtype=torch.float64), 1) if causal else None
    for b in range(B):
        for h in range(Hq):
            S = (Qf[b, h].double() @ Kf[b, h // G].double().T) * scaling
            if mask is not None:
                S = S + mask
            flags[b, :, h] = ambiguous_rows(S, delta)
    return out, flags
