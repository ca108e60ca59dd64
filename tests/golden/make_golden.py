"""Generate the golden fixtures in tests/golden/ by running the reference itself.

Run in a container where the reference checkout exists (default path below,
override with FP4_REFERENCE_DIR):

    python tests/golden/make_golden.py

The reference is imported through a shim that changes no arithmetic:

* ``nvfp4sim`` (its CUDA extension), ``lm_eval`` and ``visualize`` are
  stubbed, because fp4_quant_utils.py:13 and llama_patch.py:4,17 import them
  at module load and none is needed on the torch path;
* ``single_nvfp4_fake_quant`` / ``dual_nvfp4_fake_quant``, which
  llama_patch.py:94,96 calls but fp4_quant_utils.py only has as comments
  (:322-335), are aliased to the live ``single_nvfp4`` / ``dual_nvfp4``
  (fp4_quant_utils.py:307,336) cast back to the input dtype;
* the per-call ``print`` in single_nvfp4_quant_dequant_fused (:115) is
  silenced.

Outputs (committed): quant_torch.npz (quantizer cases), attention.npz (small
simulated-FP4 attention cases, fp32 simulation), attention_bf16.npz (the same
attention as the reference ships it for a bf16 model: bf16 quantizer, bf16
S and P), and config1.json (hash of the full [4096,4096] config-1 output).
"""
from __future__ import annotations

import contextlib
import hashlib
import io
import json
import os
import sys
import types

import numpy as np
import torch

REF = os.environ.get("FP4_REFERENCE_DIR", "/root/reference")
HERE = os.path.dirname(os.path.abspath(__file__))


def import_reference():
    sys.path.insert(0, REF)
    sys.modules.setdefault("nvfp4sim", types.ModuleType("nvfp4sim"))
    lm = types.ModuleType("lm_eval")
    lm.simple_evaluate = None
    sys.modules.setdefault("lm_eval", lm)
    vis = types.ModuleType("visualize")
    vis.collect_qkv = vis.collect_qkv_diff = lambda *a, **k: None
    sys.modules.setdefault("visualize", vis)
    import fp4_quant_utils as fqu  # noqa: E402
    import llama_patch as lp  # noqa: E402

    class Quantizer(fqu.FP4Quantizer):
        def single_nvfp4_quant_dequant_fused(self, x, global_scale_aligned=True):
            with contextlib.redirect_stdout(io.StringIO()):
                return super().single_nvfp4_quant_dequant_fused(x, global_scale_aligned)

        def single_nvfp4_fake_quant(self, x, global_scale_aligned=True):
            return self.single_nvfp4(x, global_scale_aligned).to(x.dtype)

        def dual_nvfp4_fake_quant(self, x, global_scale_aligned=True):
            return self.dual_nvfp4(x, global_scale_aligned).to(x.dtype)

    return Quantizer, lp


def quant_cases():
    """(name, tensor, input dtype) cases covering shapes, padding and edges."""
    g = torch.Generator().manual_seed(0)
    out = []
    for (m, n) in [(4, 16), (3, 37), (6, 4053), (33, 128), (1, 1), (5, 15), (128, 256)]:
        x = torch.randn(m, n, generator=g)
        idx = torch.randperm(x.numel(), generator=g)[: max(1, x.numel() // 50)]
        x.view(-1)[idx] *= 50
        out.append((f"randn_{m}x{n}", x))
    e = torch.zeros(6, 32)
    e[0, :16] = -0.0
    e[1] = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 4)  # E2M1 ties
    e[2, 3] = -1e-30
    e[3] = torch.linspace(-3, 3, 32)
    e[4] = -torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 4) * 0.125
    e[5, :16] = 448.0 * 6  # scale saturation boundary without a global scale
    e[5, 16:] = 464.0 * 6 + 1.0
    out.append(("edges", e))
    nan = torch.randn(3, 32, generator=g)
    nan[0, 5] = float("nan")
    nan[1, 7] = float("inf")
    nan[2, 0] = -float("inf")
    out.append(("nonfinite", nan))
    tiny = torch.randn(4, 48, generator=g) * 1e-3
    tiny[0, :16] *= 1e-6
    out.append(("tiny", tiny))
    out.append(("big", torch.randn(4, 32, generator=g) * 1e4))
    return out


FULL_LIMIT = 4096  # outputs with more elements are stored as a SHA-256 of their bits


def canonical_bits(y: np.ndarray) -> np.ndarray:
    """fp32 bits with every NaN replaced by 0x7FC00000 (payload and sign are not compared)."""
    y = np.ascontiguousarray(y, dtype=np.float32)
    bits = y.view(np.uint32).copy()
    bits[np.isnan(y)] = 0x7FC00000
    return bits


def _store_y(arrays, key, y):
    bits = canonical_bits(y.float().numpy())
    if bits.size <= FULL_LIMIT:
        arrays[key + "_y"] = bits
        return None
    return hashlib.sha256(np.ascontiguousarray(bits).tobytes()).hexdigest()


def make_quant(Quantizer):
    arrays = {}
    index = []
    k = 0
    for name, x in quant_cases():
        arrays["x_" + name] = x.float().numpy()
        for in_dt in (torch.float32, torch.bfloat16):
            xin = x.to(in_dt)
            for dq_name, dq in (("float32", torch.float32), ("bfloat16", torch.bfloat16), ("float16", torch.float16)):
                for gsf in (1536, None):
                    qz = Quantizer(dequant_dtype=dq, global_sf_max=gsf)
                    for aligned in ((True, False) if gsf else (True,)):
                        y = qz.single_nvfp4_quant_dequant_fused(xin, aligned)
                        key = f"c{k}"
                        h = _store_y(arrays, key, y)
                        index.append(dict(key=key, case=name, in_dtype=str(in_dt).split(".")[-1], sha256=h,
                                          dequant_dtype=dq_name, global_sf_max=gsf,
                                          gmode=("row" if aligned else "col") if gsf else "none",
                                          y_dtype=str(y.dtype).split(".")[-1]))
                        k += 1
        # dual (residual) slices, fp32 torch path
        for aligned in (True, False):
            qz = Quantizer()
            y = qz.dual_nvfp4(x, aligned)
            key = f"c{k}"
            h = _store_y(arrays, key, y)
            index.append(dict(key=key, case=name, in_dtype="float32", dequant_dtype="float32", sha256=h,
                              global_sf_max=1536, gmode="row" if aligned else "col", dual=True,
                              y_dtype=str(y.dtype).split(".")[-1]))
            k += 1
    arrays["index"] = np.frombuffer(json.dumps(index).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "quant_torch.npz"), **arrays)
    print(f"quant_torch.npz: {k} cases")


class _Mod(torch.nn.Module):
    def __init__(self, groups, quantizer):
        super().__init__()
        self.num_key_value_groups = groups
        self.fp4_quantizer = quantizer


def make_attention(Quantizer, lp):
    """Small simulated-FP4 attention cases, fp32 simulation (default dequant dtype).

    Q/K/V are fake-quantized on the 2-D views exactly as llama_patch.py:167-196
    does (Q and K row-wise, V transposed so its blocks run along tokens), then
    llama_patch.eager_attention_forward runs with the causal mask and P
    quantization on.
    """
    arrays = {}
    index = []
    lp.llama_fp4_attention_forward.quantize_enabled = True
    g = torch.Generator().manual_seed(11)
    cases = [(1, 2, 1, 256, 128, True), (2, 2, 2, 96, 128, True), (1, 2, 2, 160, 64, False), (1, 4, 2, 100, 128, True)]
    for k, (B, Hq, Hkv, T, D, causal) in enumerate(cases):
        q = torch.randn(B, Hq, T, D, generator=g).bfloat16()
        kk = torch.randn(B, Hkv, T, D, generator=g).bfloat16()
        v = torch.randn(B, Hkv, T, D, generator=g).bfloat16()
        base = f"in{k}"
        arrays[base + "_q"] = q.view(torch.int16).numpy()
        arrays[base + "_k"] = kk.view(torch.int16).numpy()
        arrays[base + "_v"] = v.view(torch.int16).numpy()
        for dual_p in (False, True):
            os.environ["FP4_USE_DUAL_QUANT_ATTN"] = "true" if dual_p else "false"
            qz = Quantizer()
            q2 = qz.single_nvfp4_fake_quant(q.permute(0, 2, 1, 3).reshape(B * T, Hq * D).float())
            k2 = qz.single_nvfp4_fake_quant(kk.permute(0, 2, 1, 3).reshape(B * T, Hkv * D).float())
            v2 = qz.single_nvfp4_fake_quant(v.permute(0, 2, 1, 3).reshape(B * T, Hkv * D).float().T,
                                            global_scale_aligned=False).T
            Qf = q2.reshape(B, T, Hq, D).permute(0, 2, 1, 3)
            Kf = k2.reshape(B, T, Hkv, D).permute(0, 2, 1, 3)
            Vf = v2.reshape(B, T, Hkv, D).permute(0, 2, 1, 3)
            mask = None
            if causal:
                mask = torch.full((T, T), float("-inf")).triu(1)[None, None].expand(B, 1, T, T)
            o, _ = lp.eager_attention_forward(_Mod(Hq // Hkv, qz), Qf, Kf, Vf, mask, scaling=D ** -0.5)
            key = f"a{len(index)}"
            arrays[key + "_o"] = o.float().numpy()
            index.append(dict(key=key, inputs=base, B=B, Hq=Hq, Hkv=Hkv, T=T, D=D, causal=causal, dual_p=dual_p))
    os.environ.pop("FP4_USE_DUAL_QUANT_ATTN", None)
    arrays["index"] = np.frombuffer(json.dumps(index).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **arrays)
    print(f"attention.npz: {len(index)} cases")


def make_attention_shipped(Quantizer, lp):
    """The reference as llama_patch.py wires it for a bf16 model (the configuration it ships with).

    FP4Quantizer(dequant_dtype=bfloat16) as llama_patch.py:126-134 builds it
    from the q_proj weight dtype; bf16 Q/K/V fake-quantized on their 2-D views
    (:167-196; single-slice Q, FP4_USE_DUAL_QUANT_Q=false); S as a bf16 matmul
    times scaling (:71) plus HF's additive bf16 causal mask (finfo(bf16).min
    above the diagonal); softmax in fp32 rounded to bf16 (:76); P fake-quant in
    bf16 (single, FP4_USE_DUAL_QUANT_ATTN=false); O = P V as a bf16 matmul
    (:102).  Outputs bf16 [B, T, Hq, D] (stored as int16 bit patterns).
    """
    arrays = {}
    index = []
    lp.llama_fp4_attention_forward.quantize_enabled = True
    os.environ["FP4_USE_DUAL_QUANT_ATTN"] = "false"
    g = torch.Generator().manual_seed(12)
    cases = [(1, 2, 1, 256, 128, True), (2, 2, 2, 96, 128, True), (1, 4, 2, 100, 128, True),
             (1, 8, 2, 384, 128, True), (1, 2, 2, 160, 128, False)]
    bf = torch.bfloat16
    for k, (B, Hq, Hkv, T, D, causal) in enumerate(cases):
        q = torch.randn(B, Hq, T, D, generator=g).bfloat16()
        kk = torch.randn(B, Hkv, T, D, generator=g).bfloat16()
        v = torch.randn(B, Hkv, T, D, generator=g).bfloat16()
        base = f"s{k}"
        arrays[base + "_q"] = q.view(torch.int16).numpy()
        arrays[base + "_k"] = kk.view(torch.int16).numpy()
        arrays[base + "_v"] = v.view(torch.int16).numpy()
        qz = Quantizer(dequant_dtype=bf)
        q2 = qz.single_nvfp4_fake_quant(q.permute(0, 2, 1, 3).reshape(B * T, Hq * D))
        k2 = qz.single_nvfp4_fake_quant(kk.permute(0, 2, 1, 3).reshape(B * T, Hkv * D))
        v2 = qz.single_nvfp4_fake_quant(v.permute(0, 2, 1, 3).reshape(B * T, Hkv * D).T,
                                        global_scale_aligned=False).T
        assert q2.dtype == k2.dtype == v2.dtype == bf
        Qf = q2.reshape(B, T, Hq, D).permute(0, 2, 1, 3)
        Kf = k2.reshape(B, T, Hkv, D).permute(0, 2, 1, 3)
        Vf = v2.reshape(B, T, Hkv, D).permute(0, 2, 1, 3)
        mask = None
        if causal:
            mask = torch.zeros(T, T, dtype=bf).masked_fill(torch.ones(T, T, dtype=torch.bool).triu(1),
                                                           torch.finfo(bf).min)[None, None].expand(B, 1, T, T)
        o, _ = lp.eager_attention_forward(_Mod(Hq // Hkv, qz), Qf, Kf, Vf, mask, scaling=D ** -0.5)
        assert o.dtype == bf
        arrays[base + "_o"] = o.contiguous().view(torch.int16).numpy()
        index.append(dict(key=base, B=B, Hq=Hq, Hkv=Hkv, T=T, D=D, causal=causal))
    os.environ.pop("FP4_USE_DUAL_QUANT_ATTN", None)
    arrays["index"] = np.frombuffer(json.dumps(index).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "attention_bf16.npz"), **arrays)
    print(f"attention_bf16.npz: {len(index)} cases")


def tiny_llama(torch_mod=torch):
    """The 2-layer random Llama of the logits fixture (4 query / 2 KV heads, head_dim 128), bf16 weights N(0, 0.02)."""
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


def make_llama_logits(Quantizer, lp):
    """Logits of the reference's patched Llama (llama_patch.py:108-250 installed as eval.py:176-179 does,
    quantization on, single-slice Q and P) on the tiny bf16 model, and of the stock model, for the
    post-RoPE drop-in's logit-level comparison.

    Shim (no arithmetic change): llama_patch.py:129-141 builds FP4Quantizer with keyword arguments
    the shipped fp4_quant_utils.py does not take (global_sf, use_search) and moves a global_sf tensor;
    the stand-in accepts them and holds that tensor.
    """
    from transformers.models.llama import modeling_llama

    class PatchQuantizer(Quantizer):
        def __init__(self, *a, global_sf=0.5, use_search=False, **kw):
            super().__init__(*a, **kw)
            self.global_sf = torch.tensor(global_sf)

    model, ids = tiny_llama()
    with torch.no_grad():
        stock = model(ids, use_cache=False).logits.float()
    os.environ["FP4_USE_DUAL_QUANT_Q"] = "false"
    os.environ["FP4_USE_DUAL_QUANT_ATTN"] = "false"
    lp.FP4Quantizer = PatchQuantizer
    lp.llama_fp4_attention_forward.quantize_enabled = True
    orig = modeling_llama.LlamaAttention.forward
    modeling_llama.LlamaAttention.forward = lp.llama_fp4_attention_forward
    try:
        with torch.no_grad():
            fp4 = model(ids, use_cache=False).logits.float()
    finally:
        modeling_llama.LlamaAttention.forward = orig
        os.environ.pop("FP4_USE_DUAL_QUANT_Q", None)
        os.environ.pop("FP4_USE_DUAL_QUANT_ATTN", None)
    np.savez_compressed(os.path.join(HERE, "llama_logits.npz"), ref_fp4=fp4.numpy(), stock=stock.numpy(),
                        ids=ids.numpy())
    cos = torch.nn.functional.cosine_similarity(fp4.flatten(), stock.flatten(), dim=0)
    print(f"llama_logits.npz: reference FP4 vs stock logits cosine {float(cos):.6f}")


def config1_input():
    """Config 1 input: randn [4096,4096] seed 0, 0.1% of entries x50, bf16."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, 4096, generator=g)
    idx = torch.randperm(x.numel(), generator=g)[: x.numel() // 1000]
    x.view(-1)[idx] *= 50
    return x.bfloat16()


def make_config1(Quantizer):
    """Per-tensor mode: g = amax * recip(2688); fused(x * recip(g)) * g, global_sf_max=None."""
    x = config1_input()
    one = torch.tensor(1.0)
    amax = x.abs().max().float()
    g = amax * (one / torch.tensor(2688.0))
    xs = x.float() * (one / g)
    y = Quantizer(global_sf_max=None).single_nvfp4_quant_dequant_fused(xs) * g
    h = hashlib.sha256(y.numpy().view(np.uint32).tobytes()).hexdigest()
    info = dict(shape=[4096, 4096], amax=float(amax), g=float(g), sha256_out_f32_bits=h,
                out_head=y[:2, :16].numpy().tolist(), torch=torch.__version__)
    with open(os.path.join(HERE, "config1.json"), "w") as f:
        json.dump(info, f, indent=1)
    print("config1.json:", h)


if __name__ == "__main__":
    # `--only NAME` regenerates one fixture file (quant, attention, attention_bf16, config1)
    only = sys.argv[sys.argv.index("--only") + 1] if "--only" in sys.argv else None
    Quantizer, lp = import_reference()
    for name, fn in (("quant", lambda: make_quant(Quantizer)), ("attention", lambda: make_attention(Quantizer, lp)),
                     ("attention_bf16", lambda: make_attention_shipped(Quantizer, lp)),
                     ("llama_logits", lambda: make_llama_logits(Quantizer, lp)),
                     ("config1", lambda: make_config1(Quantizer))):
        if only in (None, name):
            fn()
