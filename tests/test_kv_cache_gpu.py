"""NVFP4 KV cache and decode attention against the oracle.

Each call (a 300-token prefill, then single-token decode steps) quantizes its
own new tokens as the reference's patched attention does; the oracle repeats
that per call (oracle.torch_port.fake_quant_qkv) and concatenates the
results, which the cache must hold bit for bit.  Each decode output is
checked against the oracle's attention of the new token over every cached
key with the attention tolerance (attn_check).
"""
import pytest
import torch

from attn_check import DELTA, check
from oracle import torch_port as tp

pytestmark = pytest.mark.gpu

E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def _unpack(codes):
    lo, hi = (codes & 15).long(), (codes >> 4).long()
    nib = torch.stack((lo, hi), dim=-1).reshape(*codes.shape[:-1], -1)
    return E2M1[nib & 7] * torch.where((nib & 8) != 0, -1.0, 1.0)


def _e4m3(b):
    return b.view(torch.float8_e4m3fn).float()


def _dequant_cache(c):
    L = c.len
    kc, ks, kg = c.k_codes[:, :, :L].cpu(), c.k_scales[:, :, :L].cpu(), c.k_g[:, :L].cpu()
    vs, vg = c.v_scales[..., :L].cpu(), c.v_g[:, :L].cpu()
    vc = _unpack(c.v_codes.cpu())[..., :L]  # V is dim-major: [B, Hkv, D, tokens]
    k = (_unpack(kc) * _e4m3(ks).repeat_interleave(16, dim=-1)) * kg[:, None, :, None]
    v = ((vc * _e4m3(vs)) * vg[:, None, None, :]).transpose(-1, -2)
    return k, v


def _check_group_scales(c, expect_len16):
    """The per-group V scales of the prefix repeat the per-element ones."""
    L16 = c.len16
    assert L16 == expect_len16
    if L16:
        rep = c.v_scales16[..., :L16 // 16].repeat_interleave(16, dim=-1)
        assert torch.equal(rep.cpu(), c.v_scales[..., :L16].cpu())


@pytest.mark.parametrize("B,Hq,Hkv,T0,len16", [(2, 8, 2, 300, 0), (3, 4, 4, 300, 0), (1, 16, 2, 520, 512),
                                               (2, 16, 1, 700, 0), (2, 8, 2, 512, 512), (4, 32, 8, 1024, 1024),
                                               (2, 8, 2, (256, 256), 512), (2, 8, 2, (256, 200), 256)])
def test_decode_over_nvfp4_cache(B, Hq, Hkv, T0, len16):
    """Query heads per KV head 4, 1, 8 and 16; one to four splits of 256 keys; prefills whose V
    blocks are whole 16-token groups (one call, or chunks of 256) put len16 tokens of the cache
    on the group-scale path, and decode steps then extend the per-element tail."""
    from fp4_attn_b200.gemm import device_status
    from fp4_attn_b200.kv_cache import NVFP4KVCache, decode_attention
    D, steps = 128, 5
    dev = torch.device("cuda", 0)
    pre = T0 if isinstance(T0, tuple) else (T0,)
    g = torch.Generator().manual_seed(17 + B + Hq + sum(pre))
    cache = NVFP4KVCache(B, Hkv, sum(pre) + steps, D, dev)
    ks, vs = [], []

    def call(q_len):
        q = torch.randn(B, Hq, q_len, D, generator=g).bfloat16()
        k = torch.randn(B, Hkv, q_len, D, generator=g).bfloat16()
        v = torch.randn(B, Hkv, q_len, D, generator=g).bfloat16()
        cache.append(k.to(dev), v.to(dev))
        Qf, Kf, Vf = tp.fake_quant_qkv(q, k, v)
        ks.append(Kf)
        vs.append(Vf)
        return q, Qf

    for n in pre:
        call(n)
    _check_group_scales(cache, len16)
    masked = []
    for _ in range(steps):
        q, Qf = call(1)
        o = decode_attention(q.to(dev), cache).cpu()
        assert device_status() == 0
        Kf, Vf = torch.cat(ks, dim=2), torch.cat(vs, dim=2)
        kd, vd = _dequant_cache(cache)
        assert torch.equal(kd, Kf) and torch.equal(vd, Vf)  # the cache holds the reference's values
        _check_group_scales(cache, len16)
        ref = tp.eager_attention(Qf, Kf, Vf, False, D ** -0.5)  # [B, 1, Hq, D]
        G = Hq // Hkv
        flags = torch.zeros(B, 1, Hq, dtype=torch.bool)
        for b in range(B):
            for h in range(Hq):
                S = (Qf[b, h].double() @ Kf[b, h // G].double().T) * D ** -0.5
                flags[b, :, h] = tp.ambiguous_rows(S, DELTA)
        # a step has only B * Hq rows: cap it at a quarter, and the whole run near the measured 0-4.4 %
        check(o, ref, flags, max_masked_frac=0.25)
        masked.append(flags.float().mean())
    assert float(torch.stack(masked).mean()) <= 0.08
