"""Sharded long-context prefill on one GPU: every rank's slice equals the unsharded job.

The long-context prefill job (B=4, Hq=64, Hkv=8, D=128, causal, q/k/v N(0,1)*0.5
with a per-(kv-head, channel) N(0,2) bias on K, seed 2) is split by
fp4_attn_b200.shard.attention_shard over 8 ranks: a rank holds half of one
batch row's KV heads.  Each of the 8 slices is run here in turn, at a reduced
T, the way a rank runs it: the Q/K/V fake-quant covers every head of its batch
row (the reference's per-token global scales span the whole [B*T, H*D] row,
llama_patch.py:167-194) and the kernel attends only the rank's KV heads.
Checked: the packed Q/K operands and V-hat planes equal the unsharded call's
bit for bit, each slice's output equals the unsharded output's heads bit for
bit, and the assembled output meets the attention tolerance against the oracle.
"""
import pytest
import torch

from attn_check import DELTA, check
from oracle import torch_port as tp

pytestmark = pytest.mark.gpu


def _prefill_inputs(T):
    g = torch.Generator().manual_seed(2)
    B, Hq, Hkv, D = 4, 64, 8, 128
    q = (torch.randn(B, Hq, T, D, generator=g) * 0.5).bfloat16()
    k = torch.randn(B, Hkv, T, D, generator=g) * 0.5
    bias = torch.randn(Hkv, D, generator=g) * 2.0
    k = (k + bias[None, :, None, :]).bfloat16()
    v = (torch.randn(B, Hkv, T, D, generator=g) * 0.5).bfloat16()
    return q, k, v


def _rows(ws, name, b0, b1, B):
    """Rows b0..b1-1 of a workspace piece laid out by batch row (B equal slabs)."""
    t = getattr(ws, name)
    return t.reshape(B, -1)[b0:b1]


@pytest.mark.parametrize("T", [320])
def test_eight_rank_slices_equal_unsharded(T):
    from fp4_attn_b200 import shard
    from fp4_attn_b200.attention import AttentionWorkspace, fp4_attention_fwd
    from fp4_attn_b200.gemm import device_status
    q, k, v = _prefill_inputs(T)
    B, Hq, _, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    dev = torch.device("cuda", 0)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    ws_full = AttentionWorkspace(B, Hq, Hkv, T, D, dev)
    full = fp4_attention_fwd(qd, kd, vd, causal=True, workspace=ws_full)
    torch.cuda.synchronize()
    assert device_status() == 0
    parts = {}
    for r in range(8):
        units = shard.attention_shard(B, Hq, Hkv, 8, r)
        rows, (h0, h1) = shard.shard_rows(units)
        b0, b1 = rows.start, rows.stop
        ws = AttentionWorkspace(b1 - b0, Hq, Hkv, T, D, dev)
        o = fp4_attention_fwd(qd[b0:b1], kd[b0:b1], vd[b0:b1], causal=True, workspace=ws, kv_heads=(h0, h1))
        torch.cuda.synchronize()
        assert device_status() == 0
        assert o.shape == (b1 - b0, T, (h1 - h0) * G, D)
        for name in ("qc", "qs", "gq", "kc", "ks", "gk", "vhi", "vlo"):
            want = _rows(ws_full, name, b0, b1, B)
            got = getattr(ws, name).reshape(b1 - b0, -1)
            assert torch.equal(got.view(torch.uint8), want.view(torch.uint8)), f"rank {r}: packed {name} differs"
        assert torch.equal(o, full[b0:b1, :, h0 * G:h1 * G]), f"rank {r}: output differs from the unsharded call"
        for u in units:
            parts[(u.b, u.hk)] = o[u.b - b0, :, (u.hk - h0) * G:(u.hk - h0 + 1) * G].cpu()
    out = shard.assemble_attention(parts, B, T, Hq, Hkv, D)
    ref, flags = tp.attention_with_margins(q, k, v, True, D ** -0.5, delta=DELTA)
    check(out, ref, flags)


def test_kv_heads_argument_validation():
    from fp4_attn_b200.attention import fp4_attention_fwd
    dev = torch.device("cuda", 0)
    q = torch.zeros(1, 8, 128, 128, device=dev, dtype=torch.bfloat16)
    k = torch.zeros(1, 2, 128, 128, device=dev, dtype=torch.bfloat16)
    for bad in ((1, 1), (-1, 1), (0, 3)):
        with pytest.raises(ValueError):
            fp4_attention_fwd(q, k, k, kv_heads=bad)
    o = fp4_attention_fwd(q, k, k, kv_heads=(1, 2))
    assert o.shape == (1, 128, 4, 128)
