"""FP4 attention inside the Hugging Face Llama attention module.

Mirror of the reference's patch (llama_patch.py:108-250, installed by
eval.py:176-179 over transformers' LlamaAttention.forward) on the B200
kernels:

* ``fp4_eager_attention(module, query, key, value, attention_mask, scaling,
  dropout=0.0, **kw) -> (out [B, T, Hq, D], None)`` is the attention
  interface of llama_patch.eager_attention_forward (llama_patch.py:57-105)
  with the Q/K/V and P fake-quant: the tcgen05 FP4 attention kernel.  P is
  never materialised, so the weights slot is None.
* ``llama_fp4_attention_forward`` is a drop-in LlamaAttention.forward
  (transformers 5.x signature): projections, RoPE, the KV-cache update,
  ``fp4_eager_attention``, o_proj.  With a cache it also keeps, per layer,
  an NVFP4 copy of the cached K/V (``kv_cache.NVFP4KVCache``, attached to the
  HF cache object), built at the first one-token call from the prefill's
  tokens; every call's tokens are quantized as that call of the reference
  quantizes them (llama_patch.py:167-196, 212-215), and one-token calls
  (generation) attend over it with ``decode_attention``.
* ``install()`` / ``uninstall()`` swap it in and out like eval.py does.
* Single- or dual-slice Q and P follow FP4_USE_DUAL_QUANT_Q and
  FP4_USE_DUAL_QUANT_ATTN as the reference reads them (llama_patch.py:84,183:
  unset means dual).

Semantics that differ from the reference, by design:

* Q/K/V are quantized after RoPE.  The reference quantizes before RoPE
  (llama_patch.py:167-210) and applies RoPE to the dequantized values, which
  leaves them off the FP4 grid; QK^T on FP4 tensor cores needs FP4
  operands, so the native path quantizes the rotated Q and K.
* The quantizer arithmetic is fp32 (the FP4Quantizer default) whatever the
  model dtype; the reference uses the weight dtype (llama_patch.py:126-134).
* Calls are a prefill (query and key lengths equal) or one new token over
  the cache; several new tokens over a non-empty cache (chunked prefill)
  raise.  The attention mask must be causal without padding.
"""
from __future__ import annotations

import os
import weakref

import torch

from .attention import fp4_attention_fwd

_ORIGINAL = None


def dual_enabled(name: str) -> bool:
    """The reference's reading of its dual-slice switches (llama_patch.py:84,183):
    os.getenv(name, 'true').lower() == 'true' -- unset means dual."""
    return os.getenv(name, "true").lower() == "true"


# The last mask found to be plain causal: (weak reference to the tensor, its version counter, T, S).
# A model passes one mask object to every layer, so it is checked once per forward.
_CHECKED = (None, -1, 0, 0)


def _check_mask(mask: torch.Tensor | None, T: int, S: int) -> None:
    global _CHECKED
    if mask is None:
        return
    ref, version, t0, s0 = _CHECKED
    if ref is not None and ref() is mask and mask._version == version and (t0, s0) == (T, S):
        return
    if mask.dim() != 4 or mask.shape[-2] != T or mask.shape[-1] < S:
        raise ValueError(f"attention mask of shape {tuple(mask.shape)} does not match T={T}, S={S}")
    m = mask[..., :S]
    if m.dtype == torch.bool:
        allowed = m
    else:
        allowed = m > torch.finfo(m.dtype).min / 2
    # the T queries are the last T of the S positions: query i sees keys 0 .. i + S - T
    causal = torch.ones(T, S, dtype=torch.bool, device=m.device).tril(S - T)
    if not bool((allowed == causal).all()):
        raise NotImplementedError("the FP4 attention kernel supports a plain causal mask (no padding)")
    _CHECKED = (weakref.ref(mask), mask._version, T, S)


def fp4_eager_attention(module, query, key, value, attention_mask, scaling, dropout=0.0, **kwargs):
    """eager_attention_forward (llama_patch.py:57-105) on the FP4 kernel: ([B, T, Hq, D], None).

    Takes the unquantized post-RoPE query/key/value: the Q/K/V fake-quant of
    llama_patch.py:183-196 runs inside the kernel call, with dual-slice Q and P
    as FP4_USE_DUAL_QUANT_Q / FP4_USE_DUAL_QUANT_ATTN say (both dual when unset,
    as in the reference).
    """
    if dropout and getattr(module, "training", False):
        raise NotImplementedError("attention dropout is not supported")
    B, Hq, T, D = query.shape
    S = key.shape[2]
    if S != T:
        raise NotImplementedError(f"prefill only: query length {T} != key length {S}")
    _check_mask(attention_mask, T, S)
    out_dtype = torch.bfloat16 if query.dtype == torch.bfloat16 else torch.float32
    out = fp4_attention_fwd(query, key, value, causal=True, scaling=float(scaling),
                            dual_q=dual_enabled("FP4_USE_DUAL_QUANT_Q"), dual_p=dual_enabled("FP4_USE_DUAL_QUANT_ATTN"),
                            out_dtype=out_dtype)
    return out.to(query.dtype), None


# the attention call used by llama_fp4_attention_forward (tests may wrap it)
attention_interface = fp4_eager_attention


def fp4_decode_attention(module, query, cache, attention_mask, scaling):
    """One new token per sequence over the layer's NVFP4 cache (llama_patch.py:212-215 then :57-105):
    query [B, Hq, 1, D] post-RoPE -> [B, 1, Hq, D] in query's dtype."""
    from .kv_cache import decode_attention
    _check_mask(attention_mask, 1, cache.len)
    return decode_attention(query, cache, scaling=float(scaling)).to(query.dtype)


# the decode call used by llama_fp4_attention_forward (tests may wrap it)
decode_interface = fp4_decode_attention


def nvfp4_cache(past_key_values, layer_idx: int, k: torch.Tensor):
    """The layer's NVFP4 K/V cache kept beside an HF cache object (created empty on first use).
    k: the new tokens' keys [B, Hkv, T, D] (shape and device)."""
    from .kv_cache import NVFP4KVCache
    caches = getattr(past_key_values, "_fp4_attn_nvfp4", None)
    if caches is None:
        caches = {}
        past_key_values._fp4_attn_nvfp4 = caches
    c = caches.get(layer_idx)
    if c is None:
        B, Hkv, T, D = k.shape
        c = NVFP4KVCache(B, Hkv, max(T, 1) + 256, D, k.device)
        caches[layer_idx] = c
    return c


def llama_fp4_attention_forward(self, hidden_states, position_embeddings=None, attention_mask=None,
                                past_key_values=None, **kwargs):
    """LlamaAttention.forward with FP4 attention (llama_patch.py:108-250, post-RoPE quantization)."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb

    if "past_key_value" in kwargs and past_key_values is None:  # older transformers keyword
        past_key_values = kwargs.pop("past_key_value")
    input_shape = hidden_states.shape[:-1]
    hidden_shape = (*input_shape, -1, self.head_dim)
    q = self.q_proj(hidden_states).view(hidden_shape).transpose(1, 2)
    k = self.k_proj(hidden_states).view(hidden_shape).transpose(1, 2)
    v = self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
    cos, sin = position_embeddings
    q, k = apply_rotary_pos_emb(q, k, cos, sin)
    # llama_patch.py:228-232 (one host read for the three tensors)
    if bool(torch.isnan(q).any() | torch.isnan(k).any() | torch.isnan(v).any()):
        raise FloatingPointError("NaN in the attention inputs")
    T = q.shape[2]
    if past_key_values is not None:
        past = past_key_values.get_seq_length(self.layer_idx)
        if past and T != 1:
            raise NotImplementedError(f"{T} new tokens over a cache of {past}: chunked prefill is not implemented")
        k_all, v_all = past_key_values.update(k, v, self.layer_idx)  # HF's own bookkeeping (lengths, positions)
        if past:
            cache = nvfp4_cache(past_key_values, self.layer_idx, k)
            if cache.len == 0:  # the first decode step: the prefill call's tokens, quantized as that one call
                cache.grow(past + 256)
                cache.append(k_all[:, :, :past], v_all[:, :, :past])
            if cache.len != past:
                raise RuntimeError(f"NVFP4 cache holds {cache.len} tokens, the HF cache {past}")
            if cache.len + 1 > cache.capacity:
                cache.grow(2 * cache.capacity)
            cache.append(k, v)  # this call's own token
            out = decode_interface(self, q, cache, attention_mask, self.scaling)
            out = out.reshape(*input_shape, -1).contiguous()
            return self.o_proj(out), None
        k, v = k_all, v_all
    out, weights = attention_interface(self, q, k, v, attention_mask, scaling=self.scaling,
                                       dropout=0.0 if not self.training else self.attention_dropout)
    out = out.reshape(*input_shape, -1).contiguous()
    return self.o_proj(out), weights


def install() -> None:
    """Route transformers' LlamaAttention.forward to the FP4 path (eval.py:176-179)."""
    global _ORIGINAL
    from transformers.models.llama import modeling_llama

    if _ORIGINAL is None:
        _ORIGINAL = modeling_llama.LlamaAttention.forward
    modeling_llama.LlamaAttention.forward = llama_fp4_attention_forward


def uninstall() -> None:
    global _ORIGINAL
    from transformers.models.llama import modeling_llama

    if _ORIGINAL is not None:
        modeling_llama.LlamaAttention.forward = _ORIGINAL
        _ORIGINAL = None
