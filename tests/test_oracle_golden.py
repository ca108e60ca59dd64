"""The CPU oracle against golden vectors produced by the reference itself."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from oracle import quant as oq
from oracle import torch_port as tp

GOLD = os.path.join(os.path.dirname(__file__), "golden")
DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def _load(name):
    z = np.load(os.path.join(GOLD, name))
    return z, json.loads(bytes(z["index"]).decode())


def _bits_equal(y_bits: np.ndarray, ref_bits: np.ndarray) -> bool:
    return y_bits.shape == ref_bits.shape and np.array_equal(y_bits, ref_bits)


def canonical_bits(y: np.ndarray) -> np.ndarray:
    """fp32 bits with every NaN replaced by 0x7FC00000 (payload and sign are not compared)."""
    y = np.ascontiguousarray(y, dtype=np.float32)
    bits = y.view(np.uint32).copy()
    bits[np.isnan(y)] = 0x7FC00000
    return bits


def _check(y: np.ndarray, z, c):
    bits = canonical_bits(y)
    if c["sha256"] is None:
        assert _bits_equal(bits, z[c["key"] + "_y"]), c
    else:
        assert hashlib.sha256(bits.tobytes()).hexdigest() == c["sha256"], c


QZ, QIDX = _load("quant_torch.npz")


@pytest.mark.parametrize("c", QIDX, ids=[c["key"] for c in QIDX])
def test_c_oracle_matches_reference(c):
    x = torch.from_numpy(QZ["x_" + c["case"]]).to(DT[c["in_dtype"]]).float().numpy()
    if c.get("dual"):
        hi, *_ = oq.fused_qdq(x, c["gmode"], "float32", 1536.0)
        lo, *_ = oq.fused_qdq((x - hi).astype(np.float32), c["gmode"], "float32", 1536.0)
        y = hi + lo
    else:
        y, codes, scales, g = oq.fused_qdq(x, c["gmode"], c["dequant_dtype"], c["global_sf_max"])
    _check(y, QZ, c)


@pytest.mark.parametrize("c", QIDX, ids=[c["key"] for c in QIDX])
def test_torch_port_matches_reference(c):
    x = torch.from_numpy(QZ["x_" + c["case"]]).to(DT[c["in_dtype"]])
    aligned = c["gmode"] != "col"
    if c.get("dual"):
        y = tp.dual_qdq(x, aligned)
    else:
        y = tp.fused_qdq(x, aligned, c["global_sf_max"], DT[c["dequant_dtype"]])
    _check(y.float().numpy(), QZ, c)


def test_codes_reconstruct_output():
    """q*s*g from the oracle's codes/scales reproduces its dequantized output."""
    rng = np.random.RandomState(3)
    x = (rng.standard_normal((7, 53)) * 3).astype(np.float32)
    for gmode in ("row", "col", "none"):
        out, codes, scales, g = oq.fused_qdq(x, gmode, "float32", 1536.0)
        qs = oq.decode_codes(codes, scales)[:, :53]
        if gmode == "row":
            qs = qs * g[:, None]
        elif gmode == "col":
            qs = qs * g[None, :53]
        assert np.array_equal(qs.view(np.uint32), out.view(np.uint32))


def test_config1_hash():
    """Config 1 (per-tensor scale, [4096,4096]) end to end against the reference's hash."""
    info = json.load(open(os.path.join(GOLD, "config1.json")))
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, 4096, generator=g)
    idx = torch.randperm(x.numel(), generator=g)[: x.numel() // 1000]
    x.view(-1)[idx] *= 50
    x = x.bfloat16()
    one = np.float32(1.0)
    amax = np.float32(x.abs().max().float().item())
    gt = np.float32(amax * (one / np.float32(2688.0)))
    assert float(gt) == info["g"]
    xs = (x.float().numpy() * (one / gt)).astype(np.float32)
    y, *_ = oq.fused_qdq(xs, "none", "float32", None)
    y = (y * gt).astype(np.float32)
    assert hashlib.sha256(y.view(np.uint32).tobytes()).hexdigest() == info["sha256_out_f32_bits"]


AZ, AIDX = _load("attention.npz")


def _bf16(a):
    return torch.from_numpy(a).view(torch.bfloat16)


@pytest.mark.parametrize("c", AIDX, ids=[c["key"] for c in AIDX])
def test_attention_port_matches_reference(c):
    q, k, v = (_bf16(AZ[c["inputs"] + s]) for s in ("_q", "_k", "_v"))
    o = tp.attention(q, k, v, causal=c["causal"], dual_p=c["dual_p"])
    ref = torch.from_numpy(AZ[c["key"] + "_o"])
    # Same torch ops on the same CPU build: identical up to BLAS blocking.
    assert torch.allclose(o, ref, rtol=0, atol=1e-6), (o - ref).abs().max()


def test_e4m3_cast_matches_torch():
    rng = np.random.RandomState(0)
    v = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-4, 1e-2, 1, 30, 300)]
                       + [np.arange(0, 500, 0.0625, dtype=np.float32), np.array([464.0, 464.00003, -464.0, np.nan, np.inf], np.float32)])
    t = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    o = np.array([oq.e4m3_from_f32_torch(float(a)) for a in v], dtype=np.uint8)
    assert np.array_equal(o, t)


def test_fp32_configuration_distance_from_shipped_bf16():
    """The oracle's fp32 configuration against the reference's bf16-wired outputs
    (tests/golden/attention_bf16.npz): measured cosine 0.9941-0.9952, max-abs
    0.65-4.6 x RMS -- the two configurations of the reference differ by more than
    the attention tolerance; this pins that measurement."""
    import json
    import os
    import torch
    from oracle import torch_port as tp
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "attention_bf16.npz"))
    for c in json.loads(bytes(z["index"]).decode()):
        if c["T"] > 256:
            continue  # the long case runs on the GPU test only
        q, k, v = (torch.from_numpy(z[c["key"] + s]).view(torch.bfloat16) for s in ("_q", "_k", "_v"))
        ref = torch.from_numpy(z[c["key"] + "_o"]).view(torch.bfloat16).double()
        o = tp.attention(q, k, v, c["causal"]).double()
        rms = ref.pow(2).mean().sqrt()
        cos = torch.nn.functional.cosine_similarity(o.flatten(), ref.flatten(), dim=0)
        assert 0.99 <= cos < 0.9999, c
        assert (o - ref).abs().max() / rms > 2e-2, c
