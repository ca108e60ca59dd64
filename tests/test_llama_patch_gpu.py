"""The FP4 attention inside a Hugging Face Llama on the GPU.

* A small random Llama patched with fp4_attn_b200.llama_patch: every
  layer's attention output is checked against the oracle on the same
  (post-RoPE) query/key/value, with the attention tolerance of attn_check.
* The Llama-2-7B attention shape (B=8, 32 heads, MHA, T=2048, causal):
  the kernel output of a full layer checked on a subset of heads.
"""
import pytest
import torch

from attn_check import DELTA, check
from fp4_attn_b200 import llama_patch as lp
from oracle import torch_port as tp

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dual", [False, True])
def test_patched_llama_matches_oracle_per_layer(monkeypatch, dual):
    """dual=True leaves FP4_USE_DUAL_QUANT_Q / _ATTN unset: the reference's default, dual-slice Q and P."""
    from transformers import LlamaConfig, LlamaForCausalLM
    from fp4_attn_b200.attention import fp4_attention_fwd

    for name in ("FP4_USE_DUAL_QUANT_Q", "FP4_USE_DUAL_QUANT_ATTN"):
        if dual:
            monkeypatch.delenv(name, raising=False)
        else:
            monkeypatch.setenv(name, "false")

    cfg = LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=128, vocab_size=256, max_position_embeddings=512,
                      rope_theta=10000.0, attn_implementation="eager")
    torch.manual_seed(3)
    model = LlamaForCausalLM(cfg)
    for p in model.parameters():
        torch.nn.init.normal_(p, 0.0, 0.02)
    dev = torch.device("cuda", 0)
    model = model.to(dev, torch.bfloat16).eval()
    ids = torch.randint(0, 256, (2, 256), generator=torch.Generator().manual_seed(4)).to(dev)
    results = []

    def checked(module, q, k, v, mask, scaling, dropout=0.0, **kw):
        lp._check_mask(mask, q.shape[2], k.shape[2])
        o = fp4_attention_fwd(q, k, v, causal=True, scaling=float(scaling), dual_q=dual, dual_p=dual)
        qc, kc, vc = q.float().cpu(), k.float().cpu(), v.float().cpu()
        ref, flags = tp.attention_with_margins(qc, kc, vc, True, float(scaling), delta=DELTA)
        if dual:
            ref = tp.attention(qc, kc, vc, True, float(scaling), dual_q=True, dual_p=True)
        results.append(check(o.cpu(), ref, flags))
        return o.to(q.dtype), None

    monkeypatch.setattr(lp, "attention_interface", checked)
    lp.install()
    try:
        with torch.no_grad():
            logits = model(ids).logits
    finally:
        lp.uninstall()
    assert len(results) == cfg.num_hidden_layers
    assert torch.isfinite(logits.float()).all()
    # the unwrapped path gives the same logits (same kernel, same inputs)
    lp.install()
    try:
        with torch.no_grad():
            logits2 = model(ids).logits
    finally:
        lp.uninstall()
    assert torch.equal(logits, logits2)


def test_llama2_7b_attention_shape():
    """B=8, Hq=Hkv=32, D=128, T=2048, causal: full kernel call, oracle on heads 0 and 31 of rows 0 and 7."""
    from fp4_attn_b200.attention import fp4_attention_fwd
    from fp4_attn_b200.gemm import device_status
    g = torch.Generator().manual_seed(3)
    B, H, T, D = 8, 32, 2048, 128
    q = torch.randn(B, H, T, D, generator=g).bfloat16()
    k = torch.randn(B, H, T, D, generator=g).bfloat16()
    v = torch.randn(B, H, T, D, generator=g).bfloat16()
    dev = torch.device("cuda", 0)
    o = fp4_attention_fwd(q.to(dev), k.to(dev), v.to(dev), causal=True).cpu()
    assert device_status() == 0
    assert torch.isfinite(o).all()
    Qf, Kf, Vf = tp.fake_quant_qkv(q, k, v)  # whole [B*T, H*D] views
    for b in (0, 7):
        for h in (0, 31):
            qs, ks, vs = Qf[b:b + 1, h:h + 1], Kf[b:b + 1, h:h + 1], Vf[b:b + 1, h:h + 1]
            ref = tp.eager_attention(qs, ks, vs, True, D ** -0.5)
            S = (qs[0, 0].double() @ ks[0, 0].double().T) * D ** -0.5
            S = S + torch.triu(torch.full((T, T), float("-inf"), dtype=torch.float64), 1)
            flags = tp.ambiguous_rows(S, DELTA)[None, :, None]
            check(o[b:b + 1, :, h:h + 1], ref, flags, max_masked_frac=0.08)  # 4.5-5.5 % flagged at 2048 keys
