"""FP4 attention forward (tcgen05) against the simulated-FP4 attention oracle.

Tolerance (stated for the attention output O, fp32):
  * cosine(O, O_ref) >= 0.9999 over the whole output;
  * max |O - O_ref| <= 2e-2 * RMS(O_ref) over every row whose NVFP4
    quantization of P is decided at fp32 precision: rows with a P decision
    within a relative DELTA of a rounding boundary are excluded from the
    max-abs check (they stay in the cosine), because there two correct fp32
    implementations -- including the reference against itself with another
    summation order -- legitimately round to neighbouring FP4 values.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import quant as oq
from oracle import torch_port as tp

pytestmark = pytest.mark.gpu

from attn_check import DELTA, check  # noqa: E402

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _run(q, k, v, causal):
    from fp4_attn_b200.attention import fp4_attention_fwd
    from fp4_attn_b200.gemm import device_status
    dev = torch.device("cuda", 0)
    o = fp4_attention_fwd(q.to(dev), k.to(dev), v.to(dev), causal=causal).cpu()
    assert device_status() == 0
    return o


def test_prepare_v_bit_exact():
    from fp4_attn_b200.attention import prepare_v
    dev = torch.device("cuda", 0)
    rng = np.random.RandomState(3)
    B, H, T, D = 2, 3, 100, 128
    v = torch.from_numpy(rng.standard_normal((B, H, T, D)).astype(np.float32)).bfloat16()
    Tp = 128
    vhi = torch.empty(B * H * D, Tp, dtype=torch.float16, device=dev)
    vlo = torch.empty_like(vhi)
    vhat = torch.zeros(B * H * D, Tp, device=dev)
    g = torch.empty(B * T, device=dev)
    prepare_v(v.to(dev), vhi, vlo, Tp, vhat, g)
    v2d = v.permute(0, 2, 1, 3).reshape(B * T, H * D).float()
    ref, _, _, ref_g = oq.fused_qdq(np.ascontiguousarray(v2d.T.numpy()), "col", "float32", 1536.0)
    got = vhat.cpu().reshape(B, H, D, Tp)[..., :T].permute(1, 2, 0, 3).reshape(H * D, B * T).numpy()
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
    np.testing.assert_array_equal(g.cpu().numpy().view(np.uint32), ref_g[: B * T].view(np.uint32))
    s = (vhi.float() + vlo.float()).cpu().double().reshape(B, H, D, Tp)
    assert (s[..., T:] == 0).all()
    hv = vhat.cpu().double().reshape(B, H, D, Tp)
    assert ((s - hv).abs() <= hv.abs() * 2.0 ** -21 + 1e-12).all()


@pytest.mark.parametrize("B,Hq,Hkv,T,causal", [
    (1, 2, 1, 256, True), (2, 4, 2, 200, True), (1, 2, 2, 384, False), (1, 8, 2, 512, True),
    (1, 4, 4, 130, False), (3, 2, 1, 64, True), (1, 2, 1, 1, True), (2, 4, 1, 17, False)])
def test_attention_small(B, Hq, Hkv, T, causal):
    g = torch.Generator().manual_seed(B * 1000 + Hq * 100 + T)
    q = torch.randn(B, Hq, T, 128, generator=g).bfloat16()
    k = torch.randn(B, Hkv, T, 128, generator=g).bfloat16()
    v = torch.randn(B, Hkv, T, 128, generator=g).bfloat16()
    o = _run(q, k, v, causal)
    ref, flags = tp.attention_with_margins(q, k, v, causal, delta=DELTA)
    check(o, ref, flags)


def test_attention_against_reference_goldens():
    """The reference's own outputs (tests/golden/attention.npz), single P quantization, head_dim 128."""
    z = np.load(os.path.join(GOLD, "attention.npz"))
    idx = json.loads(bytes(z["index"]).decode())
    ran = 0
    for c in idx:
        if c["dual_p"] or c["D"] != 128:
            continue
        q, k, v = (torch.from_numpy(z[c["inputs"] + s]).view(torch.bfloat16) for s in ("_q", "_k", "_v"))
        o = _run(q, k, v, c["causal"])
        _, flags = tp.attention_with_margins(q, k, v, c["causal"], delta=DELTA)
        check(o, torch.from_numpy(z[c["key"] + "_o"]), flags)
        ran += 1
    assert ran >= 3


def test_attention_llama3_8b_shape_full():
    """Config 2 at full size: B=1, Hq=32, Hkv=8, T=4096, causal, q/k/v ~ N(0,1) seed 1."""
    g = torch.Generator().manual_seed(1)
    q = torch.randn(1, 32, 4096, 128, generator=g).bfloat16()
    k = torch.randn(1, 8, 4096, 128, generator=g).bfloat16()
    v = torch.randn(1, 8, 4096, 128, generator=g).bfloat16()
    o = _run(q, k, v, True)
    ref, flags = tp.attention_with_margins(q, k, v, True, delta=DELTA)
    cos, worst = check(o, ref, flags, max_masked_frac=0.12)  # 9.4 % flagged at 4096 keys
    print(f"config2: cosine {cos:.9f}, max-abs/RMS on decided rows {worst:.3e}, masked {flags.float().mean():.4f}")


# ---------------------------------------------------------------- dual-slice Q / P
def _run_dual(q, k, v, causal, dual_q, dual_p, workspace=None):
    from fp4_attn_b200.attention import fp4_attention_fwd
    from fp4_attn_b200.gemm import device_status
    dev = torch.device("cuda", 0)
    o = fp4_attention_fwd(q.to(dev), k.to(dev), v.to(dev), causal=causal, dual_q=dual_q, dual_p=dual_p,
                          workspace=workspace).cpu()
    assert device_status() == 0
    return o


def test_attention_dual_p_against_reference_goldens():
    """The reference's own outputs with FP4_USE_DUAL_QUANT_ATTN=true (tests/golden/attention.npz), head_dim 128."""
    z = np.load(os.path.join(GOLD, "attention.npz"))
    idx = json.loads(bytes(z["index"]).decode())
    ran = 0
    for c in idx:
        if not c["dual_p"] or c["D"] != 128:
            continue
        q, k, v = (torch.from_numpy(z[c["inputs"] + s]).view(torch.bfloat16) for s in ("_q", "_k", "_v"))
        o = _run_dual(q, k, v, c["causal"], False, True)
        _, flags = tp.attention_with_margins(q, k, v, c["causal"], delta=DELTA)
        check(o, torch.from_numpy(z[c["key"] + "_o"]), flags)
        ran += 1
    assert ran >= 3


@pytest.mark.parametrize("dual_q,dual_p", [(True, False), (False, True), (True, True)])
@pytest.mark.parametrize("B,Hq,Hkv,T,causal", [(1, 4, 2, 384, True), (2, 2, 1, 200, True), (1, 2, 2, 256, False)])
def test_attention_dual_against_oracle(B, Hq, Hkv, T, causal, dual_q, dual_p):
    """Dual-slice Q and/or P (the reference's defaults) against oracle.torch_port.attention(dual_q, dual_p)."""
    g = torch.Generator().manual_seed(B * 977 + Hq * 31 + T + 7 * dual_q + 3 * dual_p)
    q = torch.randn(B, Hq, T, 128, generator=g).bfloat16()
    k = torch.randn(B, Hkv, T, 128, generator=g).bfloat16()
    v = torch.randn(B, Hkv, T, 128, generator=g).bfloat16()
    o = _run_dual(q, k, v, causal, dual_q, dual_p)
    ref = tp.attention(q, k, v, causal, dual_q=dual_q, dual_p=dual_p)
    _, flags = tp.attention_with_margins(q, k, v, causal, delta=DELTA)
    check(o, ref, flags)


@pytest.mark.parametrize("strided", [False, True])
def test_dual_q_slices_bit_exact(strided):
    """Both Q slices against the C oracle: slice 1 = row mode on Q, slice 2 = row mode on the fp32 Q - slice 1.

    strided=False takes the one-pass dual quantizer; a token stride of 129
    elements (rows not 16-byte aligned) takes the three-step path.
    """
    from fp4_attn_b200.attention import AttentionWorkspace
    B, Hq, Hkv, T, D = 2, 4, 2, 200, 128
    g = torch.Generator().manual_seed(91)
    q = (torch.randn(B, Hq, T, D + (1 if strided else 0), generator=g) * 3).bfloat16()
    k = torch.randn(B, Hkv, T, D, generator=g).bfloat16()
    v = torch.randn(B, Hkv, T, D, generator=g).bfloat16()
    dev = torch.device("cuda", 0)
    qd = q.to(dev)[..., :D]
    assert (qd.stride(2) * 2) % 16 == (2 if strided else 0)
    q = q[..., :D]
    ws = AttentionWorkspace(B, Hq, Hkv, T, D, dev, dual_q=True)
    from fp4_attn_b200.attention import fp4_attention_fwd
    from fp4_attn_b200.gemm import device_status
    fp4_attention_fwd(qd, k.to(dev), v.to(dev), causal=True, dual_q=True, workspace=ws)
    assert device_status() == 0
    q2 = q.permute(0, 2, 1, 3).reshape(B * T, Hq * D).float()
    hi, c1, s1, g1 = oq.fused_qdq(np.ascontiguousarray(q2.numpy()), "row", "float32", 1536.0)
    _, c2, s2, g2 = oq.fused_qdq(np.ascontiguousarray(q2.numpy() - hi), "row", "float32", 1536.0)
    Tp = ws.Tp
    rows = (np.arange(B)[:, None] * Tp + np.arange(T)[None, :]).reshape(-1)  # workspace row of (b, t)
    nblk = Hq * D // 16
    r = rows[:, None]
    kb = np.arange(nblk)[None, :]
    off = ((r >> 7) * (nblk // 4) + (kb >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (kb & 3)
    for qc, qs, gq, codes, scales, gl in ((ws.qc, ws.qs, ws.gq, c1, s1, g1), (ws.qc_lo, ws.qs_lo, ws.gq_lo, c2, s2, g2)):
        np.testing.assert_array_equal(qc.cpu().numpy()[rows], codes)
        np.testing.assert_array_equal(gq.cpu().numpy()[rows].view(np.uint32), gl.view(np.uint32))
        np.testing.assert_array_equal(qs.cpu().numpy()[off], scales)
    pad = np.setdiff1d(np.arange(B * Tp), rows)  # padding rows read as zeros
    assert (ws.qc_lo.cpu().numpy()[pad] == 0).all() and (ws.gq_lo.cpu().numpy()[pad] == 0).all()


def test_bf16_output_is_the_fp32_result_rounded():
    """out_dtype=bf16 (the reference's output dtype) stores the fp32 result rounded to bf16, nothing else."""
    from fp4_attn_b200.attention import fp4_attention_fwd
    from fp4_attn_b200.gemm import device_status
    g = torch.Generator().manual_seed(23)
    dev = torch.device("cuda", 0)
    q = torch.randn(2, 4, 300, 128, generator=g).bfloat16().to(dev)
    k = torch.randn(2, 2, 300, 128, generator=g).bfloat16().to(dev)
    v = torch.randn(2, 2, 300, 128, generator=g).bfloat16().to(dev)
    for dual in (False, True):
        o32 = fp4_attention_fwd(q, k, v, causal=True, dual_q=dual, dual_p=dual)
        o16 = fp4_attention_fwd(q, k, v, causal=True, dual_q=dual, dual_p=dual, out_dtype=torch.bfloat16)
        assert device_status() == 0
        assert o16.dtype == torch.bfloat16 and torch.equal(o16, o32.bfloat16())


# ---------------------------------------------------------------- row-maximum kernel, fp16 V-hat PV
def _packed_heads(ws, out, B, Hq, Hkv, T, D, row_max, flags, causal=True):
    from fp4_attn_b200 import _lib
    _lib.call("fp4attn_fwd_packed_heads", ws.qc.data_ptr(), ws.qs.data_ptr(), ws.gq.data_ptr(), None, None, None,
              ws.kc.data_ptr(), ws.ks.data_ptr(), ws.gk.data_ptr(), ws.vhi.data_ptr(), ws.vlo.data_ptr(),
              _lib.ptr(row_max), out.data_ptr(), B, Hq, Hkv, T, ws.Tp, D, 0, Hkv, 1 if causal else 0, D ** -0.5,
              flags, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("B,Hq,Hkv,T,causal", [(1, 8, 2, 1000, True), (2, 4, 1, 384, False), (1, 32, 8, 4096, True)])
def test_row_max_kernel_equals_two_pass(B, Hq, Hkv, T, causal):
    """The row-maximum kernel + the attention kernel without its max pass give the output of the two-pass
    kernel: the same MMAs, the same z and the same maxima, hence the same P-hat.  The two kernels read P-hat
    for PV from different places (shared memory, TMEM), which may sum the fp32 products of O in another
    order, so O is compared to 1e-5 x RMS rather than bit for bit; one flipped P decision would move a row
    by ~1e-3 x RMS or more."""
    from fp4_attn_b200.attention import DUAL_P, AttentionWorkspace, fp4_attention_fwd
    from fp4_attn_b200.gemm import device_status
    g = torch.Generator().manual_seed(T + 5 * Hq)
    dev = torch.device("cuda", 0)
    q = torch.randn(B, Hq, T, 128, generator=g).bfloat16().to(dev)
    k = torch.randn(B, Hkv, T, 128, generator=g).bfloat16().to(dev)
    v = torch.randn(B, Hkv, T, 128, generator=g).bfloat16().to(dev)
    ws = AttentionWorkspace(B, Hq, Hkv, T, 128, dev)
    fp4_attention_fwd(q, k, v, causal=causal, workspace=ws)  # prepares the packed operands
    for flags in (0, DUAL_P):
        a = torch.full((B, T, Hq, 128), float("nan"), device=dev)
        b = torch.full((B, T, Hq, 128), float("nan"), device=dev)
        _packed_heads(ws, a, B, Hq, Hkv, T, 128, None, flags, causal)
        _packed_heads(ws, b, B, Hq, Hkv, T, 128, ws.row_max, flags, causal)
        torch.cuda.synchronize()
        assert device_status() == 0
        rms = a.double().pow(2).mean().sqrt()
        worst = float((a.double() - b.double()).abs().max() / rms)
        assert worst <= 1e-5, f"flags {flags}: max-abs / RMS {worst}"


@pytest.mark.parametrize("B,Hq,Hkv,T,causal", [(1, 8, 2, 1000, True), (2, 4, 1, 384, False), (1, 2, 1, 100, True)])
def test_pv_fp16_small(B, Hq, Hkv, T, causal):
    """FP4ATTN_PV_FP16 (V-hat rounded once to fp16 past the first 128 queries) within the tolerance."""
    from fp4_attn_b200.attention import fp4_attention_fwd
    from fp4_attn_b200.gemm import device_status
    g = torch.Generator().manual_seed(B * 31 + T)
    q = torch.randn(B, Hq, T, 128, generator=g).bfloat16()
    k = torch.randn(B, Hkv, T, 128, generator=g).bfloat16()
    v = torch.randn(B, Hkv, T, 128, generator=g).bfloat16()
    dev = torch.device("cuda", 0)
    o = fp4_attention_fwd(q.to(dev), k.to(dev), v.to(dev), causal=causal, pv_fp16=True).cpu()
    assert device_status() == 0
    ref, flags = tp.attention_with_margins(q, k, v, causal, delta=DELTA)
    check(o, ref, flags)


def test_pv_fp16_llama3_8b_shape_full():
    """Config 2 at full size with FP4ATTN_PV_FP16; bf16 output, as the bench runs it."""
    from fp4_attn_b200.attention import fp4_attention_fwd
    from fp4_attn_b200.gemm import device_status
    g = torch.Generator().manual_seed(1)
    q = torch.randn(1, 32, 4096, 128, generator=g).bfloat16()
    k = torch.randn(1, 8, 4096, 128, generator=g).bfloat16()
    v = torch.randn(1, 8, 4096, 128, generator=g).bfloat16()
    dev = torch.device("cuda", 0)
    o = fp4_attention_fwd(q.to(dev), k.to(dev), v.to(dev), causal=True, pv_fp16=True).cpu()
    assert device_status() == 0
    ref, flags = tp.attention_with_margins(q, k, v, True, delta=DELTA)
    cos, worst = check(o, ref, flags, max_masked_frac=0.12)
    print(f"config2 pv_fp16: cosine {cos:.9f}, max-abs/RMS on decided rows {worst:.3e}")
