"""fp4attn_forward_noalloc: the attention forward on the library's fixed workspace.

Collected last (file name) so it also runs after every other GPU test in the
same process.  Through the C ABI it is checked against fp4attn_forward with a
caller workspace on the same inputs -- bit-equal, and within the attention
tolerance of attn_check against the oracle -- on two calls in a row (the
second reuses the fixed workspace).
"""
import ctypes

import pytest
import torch

from attn_check import DELTA, check
from oracle import torch_port as tp

pytestmark = pytest.mark.gpu


def _call(fn, q, k, v, out, *extra):
    from fp4_attn_b200 import _lib
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    return getattr(_lib.load(), fn)(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.DTYPE_CODE[q.dtype], B, Hq, Hkv, T, D,
        q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
        v.stride(0), v.stride(1), v.stride(2), 1, D ** -0.5, out.data_ptr(), *extra,
        torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("B,Hq,Hkv,T", [(1, 4, 2, 300), (2, 8, 2, 512)])
def test_noalloc_matches_workspace_entry(B, Hq, Hkv, T):
    from fp4_attn_b200 import _lib
    from fp4_attn_b200.attention import AttentionWorkspace
    from fp4_attn_b200.gemm import device_status
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(11 + T)
    D = 128
    q = torch.randn(B, Hq, T, D, generator=g).bfloat16()
    k = torch.randn(B, Hkv, T, D, generator=g).bfloat16()
    v = torch.randn(B, Hkv, T, D, generator=g).bfloat16()
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    ws = AttentionWorkspace(B, Hq, Hkv, T, D, dev)
    ref_out = torch.empty(B, T, Hq, D, device=dev)
    assert _call("fp4attn_forward", qd, kd, vd, ref_out, ctypes.c_void_p(ws.ptr()), ws.nbytes) == 0
    ref, flags = tp.attention_with_margins(q, k, v, True, D ** -0.5, delta=DELTA)
    for _ in range(2):
        out = torch.full((B, T, Hq, D), float("nan"), device=dev)
        assert _call("fp4attn_forward_noalloc", qd, kd, vd, out) == 0, _lib.load().fp4attn_last_error()
        torch.cuda.synchronize()
        assert device_status() == 0
        assert torch.equal(out, ref_out)
        check(out.cpu(), ref, flags)


def test_noalloc_rejects_oversize_shape():
    from fp4_attn_b200 import _lib
    dev = torch.device("cuda", 0)
    B, Hq, Hkv, T, D = 1, 64, 8, 8192, 128  # needs far more than the fixed 32 MiB
    q = torch.empty(B, Hq, 1, D, device=dev).expand(B, Hq, T, D)
    k = torch.empty(B, Hkv, 1, D, device=dev).expand(B, Hkv, T, D)
    out = torch.empty(1, device=dev)
    assert _call("fp4attn_forward_noalloc", q, k, k, out) != 0
    assert b"fixed" in _lib.load().fp4attn_last_error()
