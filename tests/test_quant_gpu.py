"""GPU parity of the NVFP4 quantizer kernels against the CPU oracle.

Bar: bit-exact.  Dequantized values are compared as fp32 bits with NaNs
canonicalized (payload and sign of a NaN are not compared, its position is);
codes, scale bytes and global scales are compared exactly.
"""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from oracle import quant as oq
from oracle import torch_port as tp

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")
DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def canon(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = a.view(np.uint32).copy()
    b[np.isnan(a)] = 0x7FC00000
    return b


def make_inputs():
    rng = np.random.RandomState(1234)
    cases = []
    for (m, n) in [(4, 16), (3, 37), (64, 4053), (33, 128), (1, 1), (5, 15), (256, 1024), (17, 2080), (2, 9000)]:
        x = rng.standard_normal((m, n)).astype(np.float32)
        k = max(1, x.size // 50)
        x.reshape(-1)[rng.choice(x.size, k, replace=False)] *= 50
        cases.append((f"randn{m}x{n}", x))
    e = np.zeros((6, 32), np.float32)
    e[0, :16] = -0.0
    e[1] = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 4)
    e[2, 3] = -1e-30
    e[3] = np.linspace(-3, 3, 32)
    e[4] = -e[1] * 0.125
    e[5, :16] = 2688.0
    e[5, 16:] = 2785.0
    cases.append(("edges", e))
    f = rng.standard_normal((3, 48)).astype(np.float32)
    f[0, 5] = np.nan
    f[1, 7] = np.inf
    f[2, 0] = -np.inf
    cases.append(("nonfinite", f))
    cases.append(("tiny", (rng.standard_normal((4, 48)) * 1e-6).astype(np.float32)))
    cases.append(("big", (rng.standard_normal((4, 32)) * 1e4).astype(np.float32)))
    return cases


CASES = make_inputs()


@pytest.fixture(scope="module")
def dev():
    import fp4_attn_b200  # noqa: F401  (loads the library)
    return torch.device("cuda", 0)


@pytest.mark.parametrize("arith", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("gmode", ["row", "col", "none"])
@pytest.mark.parametrize("in_dt", ["float32", "bfloat16"])
def test_qdq_and_codes_bit_exact(dev, arith, gmode, in_dt):
    from fp4_attn_b200 import quant
    gsf = None if gmode == "none" else 1536.0
    for name, x in CASES:
        xt = torch.from_numpy(x).to(DT[in_dt])
        xin = xt.float().numpy()
        ref_out, ref_codes, ref_scales, ref_g = oq.fused_qdq(xin, gmode, arith, gsf)
        xd = xt.to(dev)
        out = quant.qdq(xd, gmode, gsf, DT[arith])
        assert out.dtype == DT[arith]
        np.testing.assert_array_equal(canon(out.float().cpu().numpy()), canon(ref_out), err_msg=name)
        pk = quant.quantize(xd, gmode, gsf, DT[arith])
        codes = pk.codes.cpu().numpy()
        scales = pk.scales.cpu().numpy()
        nanblk = (scales & 0x7F) == 0x7F
        # NaN blocks carry code 0 by convention on both sides
        np.testing.assert_array_equal(scales, ref_scales, err_msg=name)
        np.testing.assert_array_equal(codes, ref_codes, err_msg=name)
        if ref_g is not None:
            np.testing.assert_array_equal(canon(pk.g.cpu().numpy()), canon(ref_g), err_msg=name)
        assert nanblk.sum() == ((ref_scales & 0x7F) == 0x7F).sum()


def test_fp4quantizer_api_matches_torch_port(dev):
    from fp4_attn_b200 import FP4Quantizer
    for dq in (torch.float32, torch.bfloat16):
        qz = FP4Quantizer(dequant_dtype=dq)
        for name, x in CASES[:9]:
            xt = torch.from_numpy(x).bfloat16()
            for aligned in (True, False):
                ref = tp.fused_qdq(xt, aligned, 1536.0, dq)
                got = qz.single_nvfp4(xt.to(dev), aligned).cpu()
                np.testing.assert_array_equal(canon(got.float().numpy()), canon(ref.float().numpy()), err_msg=name)
                ref2 = tp.dual_qdq(xt.float(), aligned) if dq == torch.float32 else None
                if ref2 is not None:
                    got2 = qz.dual_nvfp4(xt.float().to(dev), aligned).cpu()
                    np.testing.assert_array_equal(canon(got2.numpy()), canon(ref2.numpy()), err_msg=name)


def test_transposed_view_column_mode(dev):
    """single_nvfp4(v2d.T, global_scale_aligned=False), the V quantization of llama_patch.py:196."""
    from fp4_attn_b200 import FP4Quantizer
    rng = np.random.RandomState(5)
    v = torch.from_numpy(rng.standard_normal((200, 256)).astype(np.float32)).bfloat16()
    ref = tp.fused_qdq(v.T, aligned=False)
    got = FP4Quantizer().single_nvfp4(v.to(dev).T, global_scale_aligned=False).cpu()
    np.testing.assert_array_equal(canon(got.numpy()), canon(ref.numpy()))


def test_tcgen05_scale_layout(dev):
    from fp4_attn_b200 import quant
    rng = np.random.RandomState(7)
    x = torch.from_numpy(rng.standard_normal((300, 520)).astype(np.float32)).to(dev)
    lin = quant.quantize(x, "row", scale_layout="linear")
    sw = quant.quantize(x, "row", scale_layout="tcgen05")
    m, nblk = lin.scales.shape
    nkb4 = (nblk + 3) // 4
    r = np.arange(m)[:, None]
    kb = np.arange(nblk)[None, :]
    off = ((r >> 7) * nkb4 + (kb >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (kb & 3)
    np.testing.assert_array_equal(sw.scales.cpu().numpy()[off], lin.scales.cpu().numpy())
    assert torch.equal(sw.codes, lin.codes)


def test_config1_full_size_matches_reference_hash(dev):
    """Config 1 ([4096,4096] bf16, per-tensor scale) hashed against the reference's own output."""
    from fp4_attn_b200 import quant
    info = json.load(open(os.path.join(GOLD, "config1.json")))
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, 4096, generator=g)
    idx = torch.randperm(x.numel(), generator=g)[: x.numel() // 1000]
    x.view(-1)[idx] *= 50
    x = x.bfloat16().to(dev)
    y = quant.qdq(x, "tensor", 2688.0, torch.float32)
    bits = canon(y.cpu().numpy())
    assert hashlib.sha256(bits.tobytes()).hexdigest() == info["sha256_out_f32_bits"]
    pk = quant.quantize(x, "tensor", 2688.0)
    assert float(pk.g.item()) == info["g"]


def test_attention_operand_view(dev):
    """The [B,H,T,D] -> [B*T, H*D] row-mode view (llama_patch.py:167) without a copy, T padded."""
    from fp4_attn_b200 import _lib
    rng = np.random.RandomState(9)
    B, H, T, D, Tp = 2, 3, 70, 128, 128
    q = torch.from_numpy(rng.standard_normal((B, H, T, D)).astype(np.float32)).bfloat16()
    q2d = q.permute(0, 2, 1, 3).reshape(B * T, H * D)
    ref_out, ref_codes, ref_scales, ref_g = oq.fused_qdq(q2d.float().numpy(), "row", "float32", 1536.0)
    qd = q.to(dev)
    nblk = H * D // 16
    codes = torch.full((B * Tp, H * D // 2), 0xAA, dtype=torch.uint8, device=dev)
    scales = torch.full((B * Tp, nblk), 0xAA, dtype=torch.uint8, device=dev)
    g = torch.full((B * Tp,), 7.0, device=dev)
    _lib.call("fp4q_quantize", qd.data_ptr(), 1, B, T, H, D, H * T * D, D, T * D, Tp, 1, 0, 1536.0,
              codes.data_ptr(), codes.shape[1], scales.data_ptr(), 0, nblk, g.data_ptr(), None, 0, 0,
              _lib.stream_of(qd))
    c = codes.cpu().numpy().reshape(B, Tp, -1)
    s = scales.cpu().numpy().reshape(B, Tp, -1)
    gg = g.cpu().numpy().reshape(B, Tp)
    np.testing.assert_array_equal(c[:, :T].reshape(B * T, -1), ref_codes)
    np.testing.assert_array_equal(s[:, :T].reshape(B * T, -1), ref_scales)
    np.testing.assert_array_equal(gg[:, :T].reshape(-1), ref_g)
    assert (c[:, T:] == 0).all() and (s[:, T:] == 0).all() and (gg[:, T:] == 0).all()


@pytest.mark.parametrize("search", [True, False])
def test_nvfp4sim_f32_matches_reference_cuda_numerics(dev, search):
    from fp4_attn_b200 import nvfp4sim
    rng = np.random.RandomState(11 + search)
    x = (rng.standard_normal((4096, 16)) * np.exp(rng.uniform(-12, 6, (4096, 1)))).astype(np.float32)
    x[0] = 0.0
    x[1, 3] = np.inf
    x[2, :] = -0.0
    x[3, 5] = np.nan  # every candidate loss is NaN: the group stays unwritten
    x[4, :] = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 2) / 6
    ref_q, ref_s = oq.cuda_to_nvf4(x, search)
    ref_q[3] = 0x1234
    ref_s[3] = 0x55
    xd = torch.from_numpy(x).to(dev)
    q = torch.zeros(4096, dtype=torch.int64, device=dev)
    s = torch.zeros(4096, dtype=torch.float8_e4m3fn, device=dev)
    q[3] = 0x1234
    s.view(torch.uint8)[3] = 0x55
    (nvfp4sim.f32_to_nvf4 if search else nvfp4sim.f32_to_nvf4_nosearch)(q, s, xd)
    np.testing.assert_array_equal(q.cpu().numpy().view(np.uint64), ref_q)
    np.testing.assert_array_equal(s.view(torch.uint8).cpu().numpy(), ref_s)
    out = torch.empty(4096, 16, device=dev)
    nvfp4sim.nvf4_to_f32(out, q, s)
    np.testing.assert_array_equal(canon(out.cpu().numpy()), canon(oq.cuda_from_nvf4(ref_q, ref_s)))
    out16 = torch.empty(4096, 16, dtype=torch.float16, device=dev)
    nvfp4sim.nvf4_to_f16(out16, q, s)
    ref16 = torch.from_numpy(oq.cuda_from_nvf4(ref_q, ref_s)).half().float().numpy()
    np.testing.assert_array_equal(canon(out16.float().cpu().numpy()), canon(ref16))


def test_nvfp4sim_f16_search(dev):
    from fp4_attn_b200 import nvfp4sim
    rng = np.random.RandomState(13)
    x = (rng.standard_normal((2048, 16)) * 3).astype(np.float16)
    ref_q, ref_s = oq.cuda_to_nvf4(x.astype(np.float32), True)
    xd = torch.from_numpy(x).to(dev)
    q = torch.zeros(2048, dtype=torch.int64, device=dev)
    s = torch.zeros(2048, dtype=torch.float8_e4m3fn, device=dev)
    nvfp4sim.f16_to_nvf4(q, s, xd)
    np.testing.assert_array_equal(q.cpu().numpy().view(np.uint64), ref_q)
    np.testing.assert_array_equal(s.view(torch.uint8).cpu().numpy(), ref_s)


def test_searched_path_api(dev):
    """FP4Quantizer.single_nvfp4(search=True) against the same glue run on the C oracle."""
    from fp4_attn_b200 import FP4Quantizer
    rng = np.random.RandomState(17)
    x = torch.from_numpy(rng.standard_normal((37, 100)).astype(np.float32))
    got = FP4Quantizer().single_nvfp4(x.to(dev), True, search=True).cpu()
    xp = torch.nn.functional.pad(x, (0, 12, 0, 1))
    g = xp.abs().amax(dim=1, keepdim=True) * (torch.tensor(1.0) / torch.tensor(1536.0))
    xs = xp * torch.where(g == 0, 0.0, torch.tensor(1.0) / g)
    q, s = oq.cuda_to_nvf4(xs.reshape(-1, 16).numpy(), True)
    rec = torch.from_numpy(oq.cuda_from_nvf4(q, s)).view(38, 112) * g
    ref = rec[:37, :100].bfloat16()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


def test_errors_are_raised_not_aborted(dev):
    from fp4_attn_b200 import nvfp4sim
    q = torch.zeros(3, dtype=torch.int64, device=dev)
    s = torch.zeros(3, dtype=torch.float8_e4m3fn, device=dev)
    x = torch.zeros(3, 16, device=dev)
    with pytest.raises(RuntimeError, match="even"):
        nvfp4sim.f32_to_nvf4(q, s, x)
    with pytest.raises(RuntimeError, match="CUDA"):
        nvfp4sim.f32_to_nvf4(q.cpu(), s, x)


def test_nvfp4sim_packed_exports(dev):
    """quantize_nvfp4 / dequantize_nvfp4 / qdq_nvfp4 agree with the C oracle and with each other."""
    from fp4_attn_b200 import nvfp4sim
    for name, x in CASES[:6]:
        xt = torch.from_numpy(x).bfloat16()
        ref_out, ref_codes, ref_scales, ref_g = oq.fused_qdq(xt.float().numpy(), "row", "float32", 1536.0)
        codes, scales, g = nvfp4sim.quantize_nvfp4(xt.to(dev), "row", 1536.0)
        np.testing.assert_array_equal(codes.cpu().numpy(), ref_codes, err_msg=name)
        np.testing.assert_array_equal(scales.cpu().numpy(), ref_scales, err_msg=name)
        y = nvfp4sim.qdq_nvfp4(xt.to(dev), "row", 1536.0)
        np.testing.assert_array_equal(canon(y.cpu().numpy()), canon(ref_out), err_msg=name)
        d = nvfp4sim.dequantize_nvfp4(codes, scales, g, xt.shape, "row")
        np.testing.assert_array_equal(canon(d.cpu().numpy()), canon(ref_out), err_msg=name)


@pytest.mark.parametrize("mode", ["row", "tensor", "none"])
def test_empty_rows(dev, mode):
    """Zero rows quantize to empty outputs without a launch error (in row mode the reference's
    single_nvfp4_quant_dequant_fused returns an empty tensor too)."""
    from fp4_attn_b200 import quant
    x = torch.zeros(0, 64, dtype=torch.bfloat16, device=dev)
    pk = quant.quantize(x, mode, 2688.0 if mode == "tensor" else 1536.0)
    torch.cuda.synchronize()
    assert pk.codes.shape == (0, 32) and pk.scales.numel() == 0
    out = quant.qdq(x, mode, 2688.0 if mode == "tensor" else 1536.0, torch.float32)
    assert out.shape == (0, 64)
