"""NVFP4 KV cache and decode attention (one new query token per sequence).

The reference's patched attention quantizes each call's new Q/K/V on their
2-D views (llama_patch.py:167-196: Q and K row mode on [B*q, H*D], V column
mode on the [Hkv*D, B*q] view), appends the dequantized K/V to the HF cache
(llama_patch.py:212-215) and attends over every cached key with P fake-quant
(llama_patch.py:57-105).  ``NVFP4KVCache`` keeps the packed NVFP4 data of
those same values -- codes, E4M3 scales and global scales -- and
``decode_attention`` runs the FP4 attention of a single new token over it on
the GPU (``fp4attn_decode`` in the C ABI).  As in the prefill path, Q and K
are taken after RoPE.

Layout (device tensors; Tmax is rounded up to a multiple of 256 so that the
decode kernels stream whole chunks of 256 keys):
  k_codes  uint8 [B, Hkv, Tmax, D/2]   E2M1 pairs, element 2k in the low nibble
  k_scales uint8 [B, Hkv, Tmax, D/16]  E4M3 block scales along head_dim
  k_g      fp32  [B, Tmax]             per-token global scale (row max)
  v_codes  uint8 [B, Hkv, D, Tmax/2]   V stored dim-major: byte j of channel d
                                       holds tokens 2j (low nibble) and 2j+1
  v_scales uint8 [B, Hkv, D, Tmax]     one E4M3 scale per element: a V block of
                                       16 runs along the tokens of the call that
                                       appended it
  v_g      fp32  [B, Tmax]             per-token global scale (column max / 1536)
  v_scales16 uint8 [B, Hkv, D, Tmax/16] the same V scales once per 16-token group,
                                       valid for the first len16 tokens

V is dim-major because the decode kernel contracts over the keys: a channel's
run of tokens is one row of the tensor-core operand (E2M1 pairs convert to
fp16 pairs in place, one group scale multiplies 16 tokens).

A call's V blocks coincide with whole 16-token groups of the cache when the
call starts on a group boundary and each sequence's tokens fill whole blocks
(q a multiple of 16, or B == 1, where the blocks simply run along the call's
tokens).  While every call so far did, the cache keeps len16 = the tokens
covered by such groups, and the decode kernels read those groups' scales
(1/16 of the per-element bytes).  Every scale is also stored per element.
"""
from __future__ import annotations

import torch

from . import _lib, quant

HEAD_DIM = 128


class NVFP4KVCache:
    def __init__(self, B: int, Hkv: int, Tmax: int, D: int, device):
        if D != HEAD_DIM:
            raise NotImplementedError(f"head_dim {D}: the decode kernel implements {HEAD_DIM}")
        self.B, self.Hkv, self.D = B, Hkv, D
        self.capacity = Tmax
        Tmax = (Tmax + 255) // 256 * 256
        self.Tmax = Tmax
        u8 = torch.uint8
        self.k_codes = torch.zeros(B, Hkv, Tmax, D // 2, dtype=u8, device=device)
        self.k_scales = torch.zeros(B, Hkv, Tmax, D // 16, dtype=u8, device=device)
        self.k_g = torch.zeros(B, Tmax, dtype=torch.float32, device=device)
        self.v_codes = torch.zeros(B, Hkv, D, Tmax // 2, dtype=u8, device=device)
        self.v_scales = torch.zeros(B, Hkv, D, Tmax, dtype=u8, device=device)
        self.v_g = torch.zeros(B, Tmax, dtype=torch.float32, device=device)
        self.v_scales16 = torch.zeros(B, Hkv, D, Tmax // 16, dtype=u8, device=device)
        self.len = 0
        self.len16 = 0

    def grow(self, capacity: int) -> None:
        """Reallocate for at least `capacity` tokens, keeping the cached ones (the HF cache grows the same way)."""
        if capacity <= self.capacity:
            return
        Tmax = (capacity + 255) // 256 * 256
        L = self.len
        for name in ("k_codes", "k_scales"):  # [B, Hkv, Tmax, x]
            old = getattr(self, name)
            new = torch.zeros(self.B, self.Hkv, Tmax, old.shape[-1], dtype=old.dtype, device=old.device)
            new[:, :, :L] = old[:, :, :L]
            setattr(self, name, new)
        for name, per, keep in (("v_codes", 2, (L + 1) // 2), ("v_scales", 1, L),
                                ("v_scales16", 16, (L + 15) // 16)):  # [B, Hkv, D, Tmax / per]
            old = getattr(self, name)
            new = torch.zeros(self.B, self.Hkv, self.D, Tmax // per, dtype=old.dtype, device=old.device)
            new[..., :keep] = old[..., :keep]
            setattr(self, name, new)
        for name in ("k_g", "v_g"):  # [B, Tmax]
            old = getattr(self, name)
            new = torch.zeros(self.B, Tmax, dtype=old.dtype, device=old.device)
            new[:, :L] = old[:, :L]
            setattr(self, name, new)
        self.capacity, self.Tmax = capacity, Tmax

    def append(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Quantize q new tokens k, v [B, Hkv, q, D] (post-RoPE K) as one call of the reference does, and store them."""
        _lib.require_cuda(k, v)
        B, H, q, D = k.shape
        if (B, H, D) != (self.B, self.Hkv, self.D) or v.shape != k.shape:
            raise ValueError("k/v must be [B, Hkv, q, D] matching the cache")
        if self.len + q > self.capacity:
            raise ValueError(f"cache holds {self.capacity} tokens")
        t0, t1 = self.len, self.len + q
        # K: row mode on the [B*q, Hkv*D] view (llama_patch.py:167,194)
        k2d = k.permute(0, 2, 1, 3).reshape(B * q, H * D)
        pk = quant.quantize(k2d, "row", 1536.0)
        self.k_codes[:, :, t0:t1] = pk.codes.view(B, q, H, D // 2).permute(0, 2, 1, 3)
        self.k_scales[:, :, t0:t1] = pk.scales.view(B, q, H, D // 16).permute(0, 2, 1, 3)
        self.k_g[:, t0:t1] = pk.g.view(B, q)
        # V: column mode on the [Hkv*D, B*q] view, blocks of 16 along the call's tokens (llama_patch.py:196)
        v2dT = v.permute(1, 3, 0, 2).reshape(H * D, B * q).contiguous()
        pv = quant.quantize(v2dT, "col", 1536.0)
        n = B * q
        npad = (n + 15) // 16 * 16
        lo, hi = pv.codes & 15, pv.codes >> 4
        nib = torch.stack((lo, hi), dim=-1).reshape(H * D, npad)[:, :n]  # [H*D, B*q]
        sc = pv.scales.repeat_interleave(16, dim=1)[:, :n]  # [H*D, B*q]
        nib = nib.view(H, D, B, q).permute(2, 0, 1, 3)  # [B, H, D, q]
        sc = sc.view(H, D, B, q).permute(2, 0, 1, 3)
        self.v_scales[..., t0:t1] = sc
        self.v_g[:, t0:t1] = pv.g[:n].view(B, q)
        t = t0
        if t % 2:  # the first token completes a byte whose low nibble an earlier call wrote
            j = t // 2
            self.v_codes[..., j] = (self.v_codes[..., j] & 0x0F) | (nib[..., 0].to(torch.uint8) << 4)
            nib, t = nib[..., 1:], t + 1
        if nib.shape[-1]:
            if nib.shape[-1] % 2:  # the high nibble of the last byte waits for the next call's first token
                nib = torch.cat((nib, torch.zeros_like(nib[..., :1])), dim=-1)
            packed = (nib[..., 0::2] | (nib[..., 1::2] << 4)).to(torch.uint8)
            self.v_codes[..., t // 2:t // 2 + packed.shape[-1]] = packed
        if self.len16 == t0 and t0 % 16 == 0 and (q % 16 == 0 or B == 1):
            # the call's blocks are the cache's groups t0/16 ... (the last one partial when q % 16 != 0,
            # its scale padded like the reference's block; the next call then starts mid-group)
            ng = (q + 15) // 16
            s16 = pv.scales[:, :B * ng].view(H, D, B, ng).permute(2, 0, 1, 3)  # [B, H, D, groups]
            self.v_scales16[..., t0 // 16:t0 // 16 + ng] = s16
            self.len16 = t0 + (q // 16) * 16 if q % 16 else t1
        self.len = t1


def decode_attention(q: torch.Tensor, cache: NVFP4KVCache, scaling: float | None = None,
                     workspace: torch.Tensor | None = None) -> torch.Tensor:
    """FP4 attention of one new token q [B, Hq, 1, D] (post-RoPE) over the cache -> fp32 [B, 1, Hq, D].

    q is fake-quantized like the reference's Q (row mode on the [B, Hq*D] view);
    the newest token is assumed to be in the cache already (append first).
    """
    _lib.require_cuda(q)
    B, Hq, one, D = q.shape
    if one != 1:
        raise NotImplementedError("decode_attention takes one query token per sequence")
    if B != cache.B or D != cache.D or Hq % cache.Hkv:
        raise ValueError("q [B, Hq, 1, D] must match the cache")
    if cache.len == 0:
        raise ValueError("empty cache")
    if scaling is None:
        scaling = D ** -0.5
    pq = quant.quantize(q.reshape(B, Hq * D), "row", 1536.0)
    need = _lib.load().fp4attn_decode_workspace_size(B, Hq, cache.len)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    out = torch.empty(B, Hq, D, dtype=torch.float32, device=q.device)
    _lib.call("fp4attn_decode_ex", pq.codes.data_ptr(), pq.scales.data_ptr(), pq.g.data_ptr(),
              cache.k_codes.data_ptr(), cache.k_scales.data_ptr(), cache.k_g.data_ptr(), cache.v_codes.data_ptr(),
              cache.v_scales.data_ptr(), cache.v_g.data_ptr(), cache.v_scales16.data_ptr(), cache.len16,
              B, Hq, cache.Hkv, D, cache.len, cache.Tmax, float(scaling), out.data_ptr(), workspace.data_ptr(),
              workspace.numel() * workspace.element_size(), _lib.stream_of(q))
    return out.view(B, 1, Hq, D)
