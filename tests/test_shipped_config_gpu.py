"""Distance of the kernel from the reference as it ships for a bf16 model.

tests/golden/attention_bf16.npz holds the reference's own outputs with
llama_patch.py's bf16 wiring: FP4Quantizer(dequant_dtype=bfloat16)
(llama_patch.py:126-134), S as a bf16 matmul (:71), softmax rounded to bf16
(:76), P fake-quant in bf16 arithmetic, bf16 P V (:102).  The kernel
implements the reference's fp32-arithmetic configuration (the FP4Quantizer
default dequant dtype; fp32 S and P) and is held to the attention tolerance
against it in the other tests.  Here its distance from the bf16 configuration
is measured and reported; measured on CPU with the reference's own functions,
the fp32 configuration itself is at cosine 0.9941-0.9952 and max-abs
0.65-4.6 x RMS from the bf16 one on these inputs (mostly from the Q/K/V
quantizer's bf16 arithmetic), so the stated bar is not met there and the
test only guards that distance from growing.
"""
import json
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_distance_from_the_shipped_bf16_configuration():
    from fp4_attn_b200.attention import fp4_attention_fwd
    from fp4_attn_b200.gemm import device_status
    z = np.load(os.path.join(GOLD, "attention_bf16.npz"))
    idx = json.loads(bytes(z["index"]).decode())
    dev = torch.device("cuda", 0)
    for c in idx:
        q, k, v = (torch.from_numpy(z[c["key"] + s]).view(torch.bfloat16) for s in ("_q", "_k", "_v"))
        ref = torch.from_numpy(z[c["key"] + "_o"]).view(torch.bfloat16).double()
        o = fp4_attention_fwd(q.to(dev), k.to(dev), v.to(dev), causal=c["causal"], out_dtype=torch.bfloat16)
        assert device_status() == 0
        o = o.cpu().double()
        rms = ref.pow(2).mean().sqrt()
        cos = float(torch.nn.functional.cosine_similarity(o.flatten(), ref.flatten(), dim=0))
        worst = float((o - ref).abs().max() / rms)
        print(f"{c['key']} B{c['B']} Hq{c['Hq']} Hkv{c['Hkv']} T{c['T']} causal={c['causal']}: "
              f"cosine {cos:.6f}, max-abs/RMS {worst:.3f}")
        assert cos >= 0.99 and worst <= 6.0
