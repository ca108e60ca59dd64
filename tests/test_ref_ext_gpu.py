"""The C restatement of the reference CUDA extension against the extension itself.

oracle/_ref/nvfp4sim_ref.so is the reference's fast_fp4 module compiled from
its own sources (oracle/build_ref.py); these tests run it on the GPU and
compare both the C oracle and this package's nvfp4sim kernels to it.
"""
import os

import numpy as np
import pytest
import torch

from oracle import quant as oq

pytestmark = pytest.mark.gpu

REF_SO = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "nvfp4sim_ref.so")


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_SO):
        pytest.skip("reference extension not built")
    from oracle import build_ref
    return build_ref.load()


def _inputs(seed):
    rng = np.random.RandomState(seed)
    x = (rng.standard_normal((8192, 16)) * np.exp(rng.uniform(-14, 7, (8192, 1)))).astype(np.float32)
    x[0] = 0.0
    x[1, 3] = np.inf
    x[2] = -0.0
    x[4] = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 2) / 6
    return x


@pytest.mark.parametrize("fn", ["f32_to_nvf4", "f32_to_nvf4_nosearch", "f16_to_nvf4"])
def test_quantize_against_reference_extension(ref, fn):
    import fp4_attn_b200.nvfp4sim as mine
    dev = torch.device("cuda", 0)
    x = _inputs(3)
    dt = torch.float16 if fn == "f16_to_nvf4" else torch.float32
    xd = torch.from_numpy(x).to(dt).to(dev)
    M = x.shape[0]
    outs = []
    for mod in (ref, mine):
        q = torch.zeros(M, dtype=torch.int64, device=dev)
        s = torch.zeros(M, dtype=torch.float8_e4m3fn, device=dev)
        getattr(mod, fn)(q, s, xd)
        torch.cuda.synchronize()
        outs.append((q.cpu().numpy().view(np.uint64), s.view(torch.uint8).cpu().numpy()))
    (rq, rs), (mq, ms) = outs
    np.testing.assert_array_equal(mq, rq)
    np.testing.assert_array_equal(ms, rs)
    oq_q, oq_s = oq.cuda_to_nvf4(xd.float().cpu().numpy(), fn != "f32_to_nvf4_nosearch")
    np.testing.assert_array_equal(oq_q, rq)
    np.testing.assert_array_equal(oq_s, rs)


def test_dequantize_against_reference_extension(ref):
    import fp4_attn_b200.nvfp4sim as mine
    dev = torch.device("cuda", 0)
    rng = np.random.RandomState(4)
    q = torch.from_numpy(rng.randint(-2**62, 2**62, size=4096, dtype=np.int64)).to(dev)
    s = torch.from_numpy(rng.randint(0, 256, size=4096).astype(np.uint8)).to(dev).view(torch.float8_e4m3fn)
    for fn, dt in (("nvf4_to_f32", torch.float32), ("nvf4_to_f16", torch.float16)):
        a = torch.empty(4096, 16, dtype=dt, device=dev)
        b = torch.empty(4096, 16, dtype=dt, device=dev)
        getattr(ref, fn)(a, q, s)
        getattr(mine, fn)(b, q, s)
        torch.cuda.synchronize()
        an, bn = a.float().cpu().numpy(), b.float().cpu().numpy()
        assert np.array_equal(np.isnan(an), np.isnan(bn))
        np.testing.assert_array_equal(np.nan_to_num(an), np.nan_to_num(bn))
