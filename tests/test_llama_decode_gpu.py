"""Generation through the patched Llama: prefill, then one token at a time over the NVFP4 cache.

llama_fp4_attention_forward keeps an NVFP4 copy of each layer's K/V beside the
HF cache; every call appends its own tokens quantized as that call of the
reference quantizes them (llama_patch.py:167-196, 212-215), and one-token
calls run decode_attention over it.  On a 2-layer random Llama (4 query / 2
KV heads, head_dim 128), a 64-token prefill of 2 sequences is followed by 4
greedy decode steps.  For every layer and step: the cache holds, bit for bit,
the concatenation of the reference's per-call fake-quantized K/V (the oracle
restatement of llama_patch.py:167-196), and the decode output meets the
attention tolerance against the oracle's attention of the new token over
those values.
"""
import pytest
import torch

from attn_check import DELTA, check
from oracle import torch_port as tp

pytestmark = pytest.mark.gpu

E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def _dequant(c):
    def unpack(codes):
        lo, hi = (codes & 15).long(), (codes >> 4).long()
        nib = torch.stack((lo, hi), dim=-1).reshape(*codes.shape[:-1], -1)
        return E2M1[nib & 7] * torch.where((nib & 8) != 0, -1.0, 1.0)

    L = c.len
    e4 = lambda b: b.view(torch.float8_e4m3fn).float()  # noqa: E731
    k = (unpack(c.k_codes[:, :, :L].cpu()) * e4(c.k_scales[:, :, :L].cpu()).repeat_interleave(16, dim=-1)) \
        * c.k_g[:, :L].cpu()[:, None, :, None]
    v = ((unpack(c.v_codes.cpu())[..., :L] * e4(c.v_scales[..., :L].cpu())) * c.v_g[:, :L].cpu()[:, None, None, :]) \
        .transpose(-1, -2)  # V is dim-major in the cache
    return k, v


def test_generation_decodes_over_the_nvfp4_cache(monkeypatch):
    from transformers import DynamicCache, LlamaConfig, LlamaForCausalLM

    from fp4_attn_b200 import kv_cache
    from fp4_attn_b200 import llama_patch as lp
    from fp4_attn_b200.gemm import device_status
    monkeypatch.setenv("FP4_USE_DUAL_QUANT_Q", "false")
    monkeypatch.setenv("FP4_USE_DUAL_QUANT_ATTN", "false")
    cfg = LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=128, vocab_size=256, max_position_embeddings=512,
                      rope_theta=10000.0, attn_implementation="eager")
    torch.manual_seed(3)
    model = LlamaForCausalLM(cfg)
    for p in model.parameters():
        torch.nn.init.normal_(p, 0.0, 0.02)
    dev = torch.device("cuda", 0)
    model = model.to(dev, torch.bfloat16).eval()
    B, T0, steps, D = 2, 64, 4, 128
    ids = torch.randint(0, 256, (B, T0), generator=torch.Generator().manual_seed(5)).to(dev)

    calls = {}  # layer -> list of (k, v) appended per call, post-RoPE
    orig_append = kv_cache.NVFP4KVCache.append

    def recording_append(self, k, v):
        calls.setdefault(self._layer, []).append((k.float().cpu(), v.float().cpu()))
        return orig_append(self, k, v)

    orig_cache = lp.nvfp4_cache

    def tagged_cache(pkv, layer_idx, k):
        c = orig_cache(pkv, layer_idx, k)
        c._layer = layer_idx
        return c

    checked, masked = [], []

    def checked_decode(module, q, cache, mask, scaling):
        o = lp.fp4_decode_attention(module, q, cache, mask, scaling)
        assert device_status() == 0
        kd, vd = _dequant(cache)
        # the reference's K/V fake-quant of each call (fake_quant_qkv's first argument only shapes Q)
        per_call = [tp.fake_quant_qkv(k, k, v)[1:] for k, v in calls[cache._layer]]
        Kf = torch.cat([kf for kf, _ in per_call], 2)
        Vf = torch.cat([vf for _, vf in per_call], 2)
        assert torch.equal(kd, Kf) and torch.equal(vd, Vf), "the NVFP4 cache differs from the reference's values"
        qc = q.float().cpu()
        Bq, Hq = qc.shape[:2]
        Qf = tp.fused_qdq(qc.reshape(Bq, Hq * D)).reshape(Bq, Hq, 1, D)  # row mode on the call's [B, Hq*D] view
        ref = tp.eager_attention(Qf, Kf, Vf, False, float(scaling))
        G = Hq // Kf.shape[1]
        flags = torch.zeros(Bq, 1, Hq, dtype=torch.bool)
        for b in range(Bq):
            for h in range(Hq):
                S = (Qf[b, h].double() @ Kf[b, h // G].double().T) * float(scaling)
                flags[b, :, h] = tp.ambiguous_rows(S, DELTA)
        checked.append(check(o.float().cpu(), ref, flags, max_masked_frac=0.25))  # B * Hq = 8 rows per call
        masked.append(float(flags.float().mean()))
        return o

    monkeypatch.setattr(kv_cache.NVFP4KVCache, "append", recording_append)
    monkeypatch.setattr(lp, "nvfp4_cache", tagged_cache)
    monkeypatch.setattr(lp, "decode_interface", checked_decode)
    lp.install()
    try:
        with torch.no_grad():
            cache = DynamicCache()
            out = model(ids, past_key_values=cache, use_cache=True)
            nxt = out.logits[:, -1:].argmax(-1)
            for _ in range(steps):
                out = model(nxt, past_key_values=cache, use_cache=True)
                assert torch.isfinite(out.logits.float()).all()
                nxt = out.logits[:, -1:].argmax(-1)
    finally:
        lp.uninstall()
    assert len(checked) == steps * cfg.num_hidden_layers
    assert sum(masked) / len(masked) <= 0.1
    assert all(len(c) == steps + 1 for c in calls.values())
    assert cache.get_seq_length() == T0 + steps
