"""NVFP4 GEMM (tcgen05 kind::mxf4nvf4) against float64 products of the decoded operands.

The products of E2M1 x UE4M3 values are exact; the tensor core accumulates
in fp32, so the tolerance is fp32 accumulation error: |err| <= 1e-5 * sum|a*b|.
"""
import numpy as np
import pytest
import torch

from oracle import quant as oq

pytestmark = pytest.mark.gpu


def _decoded(x_np, mode):
    out, codes, scales, g = oq.fused_qdq(x_np, mode, "float32", 1536.0)
    q = oq.decode_codes(codes, scales)[:, : x_np.shape[1]].astype(np.float64)
    return q, (g.astype(np.float64) if g is not None else None)


@pytest.mark.parametrize("M,N,K", [(128, 128, 256), (300, 200, 512), (1024, 512, 4096), (64, 1000, 256),
                                   (256, 384, 512), (512, 256, 1024), (4096, 2560, 512)])
def test_gemm_matches_decoded_products(M, N, K):
    from fp4_attn_b200 import quant
    from fp4_attn_b200.gemm import device_status, gemm_nvf4
    dev = torch.device("cuda", 0)
    rng = np.random.RandomState(M + N + K)
    a = (rng.standard_normal((M, K)) * np.exp(rng.uniform(-2, 2, (M, 1)))).astype(np.float32)
    b = rng.standard_normal((N, K)).astype(np.float32)
    qa = quant.quantize(torch.from_numpy(a).to(dev), "row", scale_layout="tcgen05")
    qb = quant.quantize(torch.from_numpy(b).to(dev), "row", scale_layout="tcgen05")
    c = gemm_nvf4(qa, qb).cpu().numpy().astype(np.float64)
    assert device_status() == 0
    ad, ga = _decoded(a, "row")
    bd, gb = _decoded(b, "row")
    ref = (ad @ bd.T) * ga[:, None] * gb[None, :]
    bound = (np.abs(ad) @ np.abs(bd).T) * ga[:, None] * gb[None, :] * 1e-5 + 1e-30
    err = np.abs(c - ref)
    assert (err <= bound).all(), f"max err/bound {np.max(err / bound)}"
