"""Work sharding for the NVFP4 path across the GPUs of one node.

The path partitions with no exchange on the data path:

* attention: a unit is one (batch, kv-head) pair -- the kv-head's K/V and
  the Hq/Hkv query heads of its GQA group.  Units are independent (softmax,
  the P quantization and PV are per query row).  The Q/K/V fake-quant of
  llama_patch.py:167-196 runs on whole [B*T, H*D] views: its per-token global
  scales span every head of a batch row.  So a rank quantizes every head of
  the batch rows its units touch (``shard_rows``) and attends only its own
  KV heads (``fp4_attention_fwd(..., kv_heads=...)``); a row split over two
  ranks is quantized by both, and every unit reads the operands the
  unsharded job reads;
* quantization: rows of the 2-D input.  Row, column and none global-scale
  modes need no exchange for row shards (a column shard would); tensor mode
  needs the tensor's max|x|, which each rank reduces locally and combines
  with one MAX all-reduce before quantizing (not on the quantize data path).

Each rank gets a contiguous, balanced block of units / rows.  Results come
back to rank 0 only for validation (``gather_to_rank0``).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


def balanced_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's contiguous share of n items (sizes differ by at most 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if n < 0:
        raise ValueError("negative item count")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


@dataclass(frozen=True)
class AttentionUnit:
    b: int   # batch row
    hk: int  # kv head; query heads hk*G .. hk*G+G-1


def attention_units(B: int, Hq: int, Hkv: int) -> list[AttentionUnit]:
    if Hq % Hkv:
        raise ValueError("Hq must be a multiple of Hkv")
    return [AttentionUnit(b, hk) for b in range(B) for hk in range(Hkv)]


def attention_shard(B: int, Hq: int, Hkv: int, world: int, rank: int) -> list[AttentionUnit]:
    units = attention_units(B, Hq, Hkv)
    s, e = balanced_range(len(units), world, rank)
    return units[s:e]


def shard_rows(units: list[AttentionUnit]) -> tuple[range, tuple[int, int]]:
    """The batch rows a shard's units touch and its KV-head range, for a shard that is a
    (batch rows) x (KV heads) block, as attention_shard gives for 1, 2, 4 or 8 ranks of the
    long-context prefill job.  Raises ValueError for a shard of another form."""
    if not units:
        raise ValueError("empty shard")
    bs, hs = sorted({u.b for u in units}), sorted({u.hk for u in units})
    if len(units) != len(bs) * len(hs) or bs != list(range(bs[0], bs[-1] + 1)) or \
            hs != list(range(hs[0], hs[-1] + 1)):
        raise ValueError("shard is not a (batch rows) x (KV heads) block")
    return range(bs[0], bs[-1] + 1), (hs[0], hs[-1] + 1)


def unit_inputs(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, u: AttentionUnit):
    """The [1, G, T, D] query and [1, 1, T, D] key/value slices of one unit."""
    G = q.shape[1] // k.shape[1]
    return (q[u.b:u.b + 1, u.hk * G:(u.hk + 1) * G], k[u.b:u.b + 1, u.hk:u.hk + 1], v[u.b:u.b + 1, u.hk:u.hk + 1])


def assemble_attention(parts: dict, B: int, T: int, Hq: int, Hkv: int, D: int) -> torch.Tensor:
    """Place per-unit outputs {(b, hk): [T, G, D]} into the [B, T, Hq, D] output."""
    G = Hq // Hkv
    first = next(iter(parts.values()))
    out = torch.empty(B, T, Hq, D, dtype=first.dtype, device=first.device)
    seen = set()
    for (b, hk), o in parts.items():
        out[b, :, hk * G:(hk + 1) * G] = o
        seen.add((b, hk))
    if len(seen) != B * Hkv:
        raise ValueError(f"{B * Hkv - len(seen)} attention units missing")
    return out


def row_shard(nrows: int, world: int, rank: int) -> slice:
    s, e = balanced_range(nrows, world, rank)
    return slice(s, e)


def tensor_amax(local_amax: torch.Tensor, group=None) -> torch.Tensor:
    """MAX all-reduce of per-rank max|x| (NaN wins, as torch.max does)."""
    t = local_amax.detach().clone().float().reshape(1)
    if torch.distributed.is_available() and torch.distributed.is_initialized():
        nan = torch.isnan(t).float()
        torch.distributed.all_reduce(nan, op=torch.distributed.ReduceOp.MAX, group=group)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX, group=group)
        if nan.item() > 0:
            t.fill_(float("nan"))
    return t


def gather_to_rank0(obj, group=None):
    """Validation only: every rank's object to rank 0 (others get None)."""
    if not (torch.distributed.is_available() and torch.distributed.is_initialized()):
        return [obj]
    world = torch.distributed.get_world_size(group)
    rank = torch.distributed.get_rank(group)
    out = [None] * world if rank == 0 else None
    torch.distributed.gather_object(obj, out, dst=0, group=group)
    return out
