"""The C ABI: the library loads and exports every entry point include/fp4attn.h declares.

CPU-only: argument validation is checked on calls that are rejected before
any CUDA work is issued.
"""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fp4attn.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^[A-Za-z_][\w \*]*?\b(\w+)\s*\(", text, flags=re.M)) - {"defined"})


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("fp4q_quantize", "nvfp4sim_f32_to_nvf4", "nvfp4sim_nvf4_to_f16", "fp4attn_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from fp4_attn_b200 import _lib
    L = _lib.load()
    for n in declared_functions():
        assert hasattr(L, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_version_and_error_string():
    from fp4_attn_b200 import _lib
    L = _lib.load()
    assert L.fp4attn_version() == 1
    assert isinstance(L.fp4attn_last_error(), bytes)


def test_argument_errors_are_codes_not_aborts():
    """Odd group counts and null pointers come back as FP4ATTN_ERR_ARG with a message."""
    from fp4_attn_b200 import _lib
    L = _lib.load()
    assert L.nvfp4sim_f32_to_nvf4(None, None, None, 3, None) == 1
    assert b"even" in L.fp4attn_last_error()
    assert L.nvfp4sim_nvf4_to_f32(None, None, None, 4, None) == 1
    assert b"null" in L.fp4attn_last_error()
    assert L.fp4q_quantize(None, 1, 1, 4, 1, 16, 0, 16, 0, 4, 1, 0, 1536.0, None, 0, None, 0, 0, None, None, 0, 0,
                           None) == 1
    assert L.fp4q_quantize(ctypes.c_void_p(16), 1, 1, 4, 1, 16, 0, 16, 0, 4, 1, 0, 1536.0, None, 0, None, 0, 0,
                           None, None, 0, 0, None) == 1
    assert b"g buffer" in L.fp4attn_last_error()


def test_python_api_refuses_cpu_tensors():
    import torch
    from fp4_attn_b200 import FP4Quantizer
    with pytest.raises(RuntimeError, match="CUDA"):
        FP4Quantizer().single_nvfp4(torch.randn(4, 16))


def test_attention_workspace_layout():
    """Pieces of the fp4attn_forward workspace: 256-byte aligned, in order, sized for the Llama-3-8B shape."""
    from fp4_attn_b200 import _lib
    L = _lib.load()
    offs = (ctypes.c_int64 * 8)()
    B, Hq, Hkv, T, D = 1, 32, 8, 4096, 128
    total = L.fp4attn_workspace_layout(B, Hq, Hkv, T, D, offs)
    sizes = [T * Hq * D // 2, T // 128 * Hq * 2 * 512, T * 4, T * Hkv * D // 2, T // 128 * Hkv * 2 * 512, T * 4,
             Hkv * D * T * 2, Hkv * D * T * 2]
    o = list(offs)
    assert o[0] == 0 and all(x % 256 == 0 for x in o)
    for i in range(7):
        assert o[i + 1] >= o[i] + sizes[i]
    assert total >= o[7] + sizes[7] and total % 256 == 0
    assert L.fp4attn_workspace_layout(1, 3, 2, 128, 128, None) == -1  # Hq % Hkv != 0
    assert L.fp4attn_workspace_layout(1, 2, 1, 0, 128, None) == -1


def test_attention_forward_argument_errors():
    from fp4_attn_b200 import _lib
    L = _lib.load()
    args = [None, None, None, 1, 1, 2, 1, 128, 128] + [0] * 9 + [1, 0.1, None, None, 0, None]
    assert L.fp4attn_forward(*args) == 1
    assert b"null" in L.fp4attn_last_error()
    p = ctypes.c_void_p(256)
    args = [p, p, p, 1, 1, 2, 1, 128, 128] + [0] * 9 + [1, 0.1, p, p, 16, None]
    assert L.fp4attn_forward(*args) == 1
    assert b"workspace" in L.fp4attn_last_error()


def test_decode_argument_errors():
    """fp4attn_decode rejects bad arguments with a status code before touching the device."""
    from fp4_attn_b200 import _lib
    L = _lib.load()
    assert L.fp4attn_decode_workspace_size(0, 32, 10) == -1
    B, Hq, Hkv, D, len_ = 2, 32, 8, 128, 300
    need = L.fp4attn_decode_workspace_size(B, Hq, len_)
    nsplit = (len_ + 255) // 256
    assert need == (B * Hq * nsplit * 256 + B * Hq * nsplit * (D + 4) + B * Hq) * 4
    p = ctypes.c_void_p(256)

    def call(ptr=p, Hq=Hq, Hkv=Hkv, D=D, len_=len_, Tmax=512, ws_bytes=need, ws=p):
        return L.fp4attn_decode(ptr, ptr, ptr, ptr, ptr, ptr, ptr, ptr, ptr, B, Hq, Hkv, D, len_, Tmax, 0.088,
                                ptr, ws, ws_bytes, None)

    assert call(ptr=None) == 1 and b"null" in L.fp4attn_last_error()
    assert call(D=64) == 3 and b"head_dim" in L.fp4attn_last_error()
    assert call(Tmax=299) == 1 and b"shape" in L.fp4attn_last_error()
    assert call(Tmax=400) == 1 and b"multiple of 256" in L.fp4attn_last_error()
    assert call(Hq=34, Hkv=2) == 3 and b"query heads" in L.fp4attn_last_error()
    assert call(ptr=ctypes.c_void_p(264)) == 1 and b"aligned" in L.fp4attn_last_error()
    assert call(ws_bytes=need - 4) == 1 and b"workspace" in L.fp4attn_last_error()
