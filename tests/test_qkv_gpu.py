"""Q/K projection fused with RoPE and the NVFP4 row quantizer (fp4_attn_b200.qkv) against the oracle.

* Exact case: x and W on small integer grids (x in k/8, W in k/64, |k| <= 4), so
  every product and partial sum of x W^T is exact in fp32 and the kernel's
  accumulation order cannot matter: codes, E4M3 scales and g must equal the
  oracle's bit for bit.  The oracle is the reference's own op order: the bf16
  projection, HF apply_rotary_pos_emb in bf16 (torch on CPU), then the row
  quantizer (oracle.quant.fused_qdq, fp32 arithmetic).
* Realistic case: N(0,1) hidden states and N(0,0.02) weights, the whole layer
  attention from the hidden states against oracle.torch_port on the same
  post-RoPE bf16 Q/K/V, with the attention tolerance (attn_check).
"""
import numpy as np
import pytest
import torch

from attn_check import DELTA, check
from oracle import quant as oq
from oracle import torch_port as tp

pytestmark = pytest.mark.gpu


def _rope_tables(B, T, D=128, base=10000.0):
    inv = 1.0 / (base ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    ang = torch.arange(T, dtype=torch.float32)[:, None] * inv[None, :]
    emb = torch.cat((ang, ang), dim=-1)
    cos = emb.cos().bfloat16()[None].expand(B, T, D).contiguous()
    sin = emb.sin().bfloat16()[None].expand(B, T, D).contiguous()
    return cos, sin


def _rope_bf16(y, cos, sin):
    """HF apply_rotary_pos_emb on bf16 tensors: (y * cos) + (rotate_half(y) * sin)."""
    h = y.shape[-1] // 2
    rot = torch.cat((-y[..., h:], y[..., :h]), dim=-1)
    return (y * cos) + (rot * sin)


def _atoms_to_linear(sc, M, nblk):
    r = np.arange(M)[:, None]
    kb = np.arange(nblk)[None, :]
    off = ((r >> 7) * (nblk // 4) + (kb >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (kb & 3)
    return sc[off]


@pytest.mark.parametrize("H,B,T,K", [(32, 2, 256, 1024), (8, 2, 256, 1024), (4, 2, 256, 1024), (2, 2, 256, 1024),
                                     (1, 2, 256, 1024), (32, 1, 4096, 256), (8, 4, 4096, 256)])
def test_rope_quant_projection_bit_exact(H, B, T, K):
    """The last two shapes have more tiles (token block x 4-head group) than SMs, so CTAs take
    several tiles and some token blocks' tiles run in different rounds of the persistent grid."""
    from fp4_attn_b200.gemm import device_status
    from fp4_attn_b200.qkv import rope_quant_projection
    D = 128
    g = torch.Generator().manual_seed(7 + H)
    x = (torch.randint(-4, 5, (B * T, K), generator=g).float() / 8).bfloat16()
    w = (torch.randint(-4, 5, (H * D, K), generator=g).float() / 64).bfloat16()
    cos, sin = _rope_tables(B, T, D)
    dev = torch.device("cuda", 0)
    codes, scales, gq = rope_quant_projection(x.to(dev), w.to(dev), cos.reshape(B * T, D).to(dev),
                                              sin.reshape(B * T, D).to(dev), T)
    torch.cuda.synchronize()
    assert device_status() == 0
    y = (x.double() @ w.double().T).float().bfloat16()  # exact sums, one rounding to bf16
    z = _rope_bf16(y.view(B * T, H, D), cos.reshape(B * T, 1, D), sin.reshape(B * T, 1, D)).reshape(B * T, H * D)
    _, rc, rs, rg = oq.fused_qdq(np.ascontiguousarray(z.float().numpy()), "row", "float32", 1536.0)
    np.testing.assert_array_equal(codes.cpu().numpy(), rc)
    np.testing.assert_array_equal(gq.cpu().numpy().view(np.uint32), rg.view(np.uint32))
    np.testing.assert_array_equal(_atoms_to_linear(scales.cpu().numpy(), B * T, H * D // 16), rs)


def _layer_inputs(exact, B, T, K, Hq, Hkv, D, seed):
    g = torch.Generator().manual_seed(seed)
    if exact:  # integer grids: x W^T exact in fp32 whatever the summation order
        hidden = (torch.randint(-4, 5, (B, T, K), generator=g).float() / 8).bfloat16()
        ws = [(torch.randint(-4, 5, (h * D, K), generator=g).float() / 64).bfloat16() for h in (Hq, Hkv, Hkv)]
    else:
        hidden = torch.randn(B, T, K, generator=g).bfloat16()
        ws = [(torch.randn(h * D, K, generator=g) * 0.02).bfloat16() for h in (Hq, Hkv, Hkv)]
    return hidden, ws


@pytest.mark.parametrize("exact", [True, False])
def test_attention_from_hidden_against_oracle(exact):
    """The whole layer from the hidden states against the oracle on the same post-RoPE bf16 Q/K/V.

    exact=True: the projections are exact, so the oracle sees the kernel's own
    Q/K/V and the attention tolerance applies in full.  exact=False (N(0,1)
    hidden states): the projection's fp32 summation order differs from any
    other GEMM's, which moves the last bf16 bit of some projected values and,
    near an E2M1 decision, their codes; the cosine bar still applies.
    """
    from fp4_attn_b200.gemm import device_status
    from fp4_attn_b200.qkv import attention_from_hidden
    B, T, K, Hq, Hkv, D = 1, 384, 1024, 8, 2, 128
    hidden, (wq, wk, wv) = _layer_inputs(exact, B, T, K, Hq, Hkv, D, 31)
    cos, sin = _rope_tables(B, T, D)
    dev = torch.device("cuda", 0)
    o = attention_from_hidden(hidden.to(dev), wq.to(dev), wk.to(dev), wv.to(dev), cos.to(dev), sin.to(dev),
                              out_dtype=torch.float32).cpu()
    assert device_status() == 0
    q = (hidden.double() @ wq.double().T).float().bfloat16().view(B, T, Hq, D)
    k = (hidden.double() @ wk.double().T).float().bfloat16().view(B, T, Hkv, D)
    v = (hidden.double() @ wv.double().T).float().bfloat16().view(B, T, Hkv, D).transpose(1, 2)
    q = _rope_bf16(q, cos[:, :, None], sin[:, :, None]).transpose(1, 2)
    k = _rope_bf16(k, cos[:, :, None], sin[:, :, None]).transpose(1, 2)
    ref, flags = tp.attention_with_margins(q, k, v, True, D ** -0.5, delta=DELTA)
    if exact:
        check(o, ref, flags)
    else:
        cos_sim = torch.nn.functional.cosine_similarity(o.double().flatten(), ref.double().flatten(), dim=0)
        assert cos_sim >= 0.9999, f"cosine {cos_sim}"
