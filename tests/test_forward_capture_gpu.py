"""fp4attn_forward_ex inside a CUDA-graph capture: an argument error found after the
side streams were forked still leaves the caller's capture valid.

The forward forks K quantization and V-hat preparation onto two side streams.
Here the input dtype code is invalid, which only the quantizer notices -- after
the fork.  The call must return the error and join the side streams back, so
that ending the capture succeeds (an unjoined fork invalidates it).  Nothing is
launched: the bad dtype is rejected on the host.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_late_argument_error_keeps_capture_valid():
    from fp4_attn_b200 import _lib
    from fp4_attn_b200.attention import AttentionWorkspace
    dev = torch.device("cuda", 0)
    B, Hq, Hkv, T, D = 1, 4, 2, 256, 128
    q = torch.zeros(B, Hq, T, D, device=dev, dtype=torch.bfloat16)
    k = torch.zeros(B, Hkv, T, D, device=dev, dtype=torch.bfloat16)
    out = torch.empty(B, T, Hq, D, device=dev)
    ws = AttentionWorkspace(B, Hq, Hkv, T, D, dev)
    L = _lib.load()
    st = torch.cuda.Stream(dev)
    g = torch.cuda.CUDAGraph()
    rc = None
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            rc = L.fp4attn_forward_ex(q.data_ptr(), k.data_ptr(), k.data_ptr(), 7, B, Hq, Hkv, T, D, q.stride(0),
                                      q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2), k.stride(0),
                                      k.stride(1), k.stride(2), 1, D ** -0.5, 0, out.data_ptr(), ws.ptr(), ws.nbytes,
                                      st.cuda_stream)
    assert rc != 0
    assert b"dtype" in L.fp4attn_last_error()
    g.replay()  # the captured graph holds only the fork/join event nodes
    torch.cuda.synchronize()
