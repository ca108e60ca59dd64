"""Host logic of fp4_attn_b200.llama_patch on CPU: patching, refusals, masks.

No kernel runs here: every case stops at a check before the GPU (and the
kernel path itself refuses CPU tensors -- there is no CPU fallback).
"""
import pytest
import torch

from fp4_attn_b200 import llama_patch as lp


def _tiny_model():
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=1, num_attention_heads=2,
                      num_key_value_heads=1, head_dim=128, vocab_size=64, max_position_embeddings=64,
                      attn_implementation="eager")
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).eval()


def test_install_uninstall_restores_forward():
    from transformers.models.llama import modeling_llama as M
    orig = M.LlamaAttention.forward
    lp.install()
    try:
        assert M.LlamaAttention.forward is lp.llama_fp4_attention_forward
        lp.install()  # idempotent
    finally:
        lp.uninstall()
    assert M.LlamaAttention.forward is orig


def test_dual_switches_read_as_the_reference_reads_them(monkeypatch):
    """os.getenv(name, 'true').lower() == 'true' (llama_patch.py:84,183): unset means dual."""
    for name in ("FP4_USE_DUAL_QUANT_Q", "FP4_USE_DUAL_QUANT_ATTN"):
        monkeypatch.delenv(name, raising=False)
        assert lp.dual_enabled(name)
        for v, want in (("true", True), ("TRUE", True), ("false", False), ("1", False), ("", False)):
            monkeypatch.setenv(name, v)
            assert lp.dual_enabled(name) is want


def test_patched_model_reaches_the_kernel_with_dual_defaults(monkeypatch):
    """With the switches unset the patched Llama asks the kernel for dual-slice Q and P."""
    model = _tiny_model()
    ids = torch.randint(0, 64, (1, 8))
    seen = []

    def fake(q, k, v, causal=True, scaling=None, dual_q=False, dual_p=False, out_dtype=None):
        seen.append((dual_q, dual_p))
        raise RuntimeError("stop before the GPU")

    monkeypatch.delenv("FP4_USE_DUAL_QUANT_Q", raising=False)
    monkeypatch.setenv("FP4_USE_DUAL_QUANT_ATTN", "true")
    monkeypatch.setattr(lp, "fp4_attention_fwd", fake)
    lp.install()
    try:
        with pytest.raises(RuntimeError, match="stop before"):
            model(ids)
        monkeypatch.setenv("FP4_USE_DUAL_QUANT_Q", "false")
        monkeypatch.setenv("FP4_USE_DUAL_QUANT_ATTN", "false")
        with pytest.raises(RuntimeError, match="stop before"):
            model(ids)
    finally:
        lp.uninstall()
    assert seen == [(True, True), (False, False)]


def test_cpu_tensors_are_refused():
    q = torch.randn(1, 2, 16, 128).bfloat16()
    k = torch.randn(1, 1, 16, 128).bfloat16()
    with pytest.raises(RuntimeError):
        lp.fp4_eager_attention(torch.nn.Module(), q, k, k, None, scaling=128 ** -0.5)


def test_decode_shape_is_refused():
    q = torch.randn(1, 2, 1, 128)
    k = torch.randn(1, 1, 16, 128)
    with pytest.raises(NotImplementedError):
        lp.fp4_eager_attention(torch.nn.Module(), q, k, k, None, scaling=1.0)


def test_mask_check():
    T = 8
    causal = torch.full((T, T), torch.finfo(torch.float32).min).triu(1)[None, None]
    lp._check_mask(causal, T, T)
    lp._check_mask(None, T, T)
    lp._check_mask(torch.ones(T, T, dtype=torch.bool).tril()[None, None], T, T)
    padded = causal.clone()
    padded[..., :, 0] = torch.finfo(torch.float32).min  # a padded first key
    with pytest.raises(NotImplementedError):
        lp._check_mask(padded, T, T)
    with pytest.raises(ValueError):
        lp._check_mask(causal[..., :4, :], T, T)
    # a mask already found causal is not re-read, unless it was changed in place since
    m = causal.clone()
    lp._check_mask(m, T, T)
    lp._check_mask(m, T, T)
    m[..., :, 0] = torch.finfo(torch.float32).min
    with pytest.raises(NotImplementedError):
        lp._check_mask(m, T, T)


def test_nvfp4sim_new_exports_refuse_unimplemented_modes():
    from fp4_attn_b200 import nvfp4sim
    for name in ("quantize_nvfp4", "dequantize_nvfp4", "qdq_nvfp4", "fp4_attention_fwd"):
        assert callable(getattr(nvfp4sim, name))
    q = torch.randn(1, 2, 16, 128)
    with pytest.raises(RuntimeError, match="CUDA"):  # dual modes exist; no CPU path
        nvfp4sim.fp4_attention_fwd(q, q[:, :1], q[:, :1], dual_p=True)
    with pytest.raises(NotImplementedError):
        nvfp4sim.fp4_attention_fwd(q, q[:, :1], q[:, :1], v_scale_mode="channel")
    with pytest.raises(NotImplementedError):
        nvfp4sim.quantize_nvfp4(torch.randn(4, 16), search=True)


def test_kv_cache_host_checks():
    from fp4_attn_b200 import kv_cache
    with pytest.raises(NotImplementedError):
        kv_cache.NVFP4KVCache(1, 1, 16, 64, "cpu")
    c = kv_cache.NVFP4KVCache(1, 2, 16, 128, "cpu")
    k = torch.randn(1, 2, 4, 128)
    with pytest.raises(RuntimeError, match="CUDA"):  # no CPU path
        c.append(k, k)
    with pytest.raises(RuntimeError, match="CUDA"):
        kv_cache.decode_attention(torch.randn(1, 4, 1, 128), c)


def test_mask_check_for_new_tokens_over_a_cache():
    """T new queries over S keys: query i sees keys 0 .. i + S - T (a one-token decode sees all)."""
    S = 8
    lp._check_mask(torch.zeros(1, 1, 1, S), 1, S)
    m = torch.full((2, S), torch.finfo(torch.float32).min).triu(S - 2 + 1)[None, None]
    lp._check_mask(m, 2, S)
    bad = torch.zeros(1, 1, 1, S)
    bad[..., 3] = torch.finfo(torch.float32).min
    with pytest.raises(NotImplementedError):
        lp._check_mask(bad, 1, S)


def test_kv_cache_grow_keeps_tokens():
    from fp4_attn_b200 import kv_cache
    c = kv_cache.NVFP4KVCache(2, 2, 10, 128, "cpu")
    c.k_codes[:, :, :5] = 7
    c.v_scales[..., :5] = 3  # V is dim-major: tokens along the last axis
    c.v_codes[..., :3] = 0x21
    c.k_g[:, :5] = 1.5
    c.len = 5
    c.grow(300)
    assert c.capacity == 300 and c.Tmax == 512 and c.k_codes.shape[2] == 512
    assert (c.k_codes[:, :, :5] == 7).all() and (c.k_codes[:, :, 5:] == 0).all()
    assert (c.v_scales[..., :5] == 3).all() and (c.v_scales[..., 5:] == 0).all() and c.v_scales.shape[-1] == 512
    assert (c.v_codes[..., :3] == 0x21).all() and (c.v_codes[..., 3:] == 0).all() and c.v_codes.shape[-1] == 256
    assert (c.k_g[:, :5] == 1.5).all() and (c.k_g[:, 5:] == 0).all()
