"""Logits of the patched Llama against the reference's own patched forward.

tests/golden/llama_logits.npz holds the logits of the reference's patched
attention (llama_patch.py:108-250 installed as eval.py:176-179 does,
quantization on, single-slice Q and P) on a 2-layer random bf16 Llama, and
the stock model's, computed by tests/golden/make_golden.py from the reference
itself.  The drop-in here quantizes after RoPE with fp32 quantizer arithmetic,
the reference before RoPE with bf16 arithmetic (llama_patch.py:126-134,
167-210), so the two FP4 forwards differ by design; this test reports that
deviation next to the FP4-versus-stock one and only guards it loosely.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden", "llama_logits.npz")


def _tiny_llama():
    # the model of make_golden.tiny_llama
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=128, vocab_size=256, max_position_embeddings=512,
                      rope_theta=10000.0, attn_implementation="eager")
    torch.manual_seed(3)
    model = LlamaForCausalLM(cfg)
    for p in model.parameters():
        torch.nn.init.normal_(p, 0.0, 0.02)
    ids = torch.randint(0, 256, (2, 128), generator=torch.Generator().manual_seed(4))
    return model.to(torch.bfloat16).eval(), ids


def _cmp(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    cos = float(torch.nn.functional.cosine_similarity(a, b, dim=0))
    return cos, float((a - b).abs().max() / b.pow(2).mean().sqrt())


def test_patched_logits_against_the_reference_forward(monkeypatch):
    from fp4_attn_b200 import llama_patch as lp
    z = np.load(GOLD)
    model, ids = _tiny_llama()
    assert np.array_equal(ids.numpy(), z["ids"])
    ref_fp4, stock = torch.from_numpy(z["ref_fp4"]), torch.from_numpy(z["stock"])
    monkeypatch.setenv("FP4_USE_DUAL_QUANT_Q", "false")
    monkeypatch.setenv("FP4_USE_DUAL_QUANT_ATTN", "false")
    dev = torch.device("cuda", 0)
    model = model.to(dev)
    lp.install()
    try:
        with torch.no_grad():
            ours = model(ids.to(dev), use_cache=False).logits.float().cpu()
    finally:
        lp.uninstall()
    assert torch.isfinite(ours).all()
    c_ref, e_ref = _cmp(ours, ref_fp4)
    c_stock, e_stock = _cmp(ref_fp4, stock)
    c_ours_stock, _ = _cmp(ours, stock)
    print(f"patched logits vs the reference's patched forward: cosine {c_ref:.6f}, max-abs/RMS {e_ref:.4f}; "
          f"reference FP4 vs stock: cosine {c_stock:.6f}, max-abs/RMS {e_stock:.4f}; ours vs stock: cosine "
          f"{c_ours_stock:.6f}")
    assert c_ref >= 0.999
