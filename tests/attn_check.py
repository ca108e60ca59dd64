"""Attention output check shared by the GPU attention tests.

Tolerance (stated for the attention output O, fp32):
  * cosine(O, O_ref) >= 0.9999 over the whole output;
  * max |O - O_ref| <= 2e-2 * RMS(O_ref) over every row whose NVFP4
    quantization of P is decided at fp32 precision (rows flagged by
    oracle.torch_port.ambiguous_rows at relative DELTA are excluded from the
    max-abs check and stay in the cosine).

The masked fraction is capped near what the oracle flags on the tests'
inputs, so a regression that moves many rows cannot hide behind the mask:
rows of up to a few hundred keys flag at most 1.6 % (cap 5 %), rows of 2048
keys 4.5-5.5 %, 4096 keys 9.4 % (callers with long rows pass their own cap).
"""
import torch

DELTA = 1e-5


def check(o_gpu, o_ref, flags=None, max_masked_frac=0.05):
    o_gpu, o_ref = o_gpu.double(), o_ref.double()
    rms = o_ref.pow(2).mean().sqrt()
    cos = torch.nn.functional.cosine_similarity(o_gpu.flatten(), o_ref.flatten(), dim=0)
    assert cos >= 0.9999, f"cosine {cos}"
    err = (o_gpu - o_ref).abs().amax(-1)  # per (b, t, h) row
    ok = torch.ones_like(err, dtype=torch.bool) if flags is None else ~flags
    if flags is not None:
        assert flags.float().mean() <= max_masked_frac, f"masked fraction {flags.float().mean()}"
    worst = err[ok].max() / rms
    assert worst <= 2e-2, f"max-abs / RMS on decided rows = {worst}"
    return float(cos), float(worst)
