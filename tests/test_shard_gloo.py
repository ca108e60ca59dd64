"""Multi-rank host logic of fp4_attn_b200.shard on CPU (gloo, world size 2).

The per-rank compute here is the oracle (test infrastructure); on a GPU node
the same plan drives the CUDA kernels.  The checks: every unit / row is
owned by exactly one rank, the sharded results reassemble to the unsharded
ones bit for bit, and the tensor-mode max reduction equals the global max
(NaN included).
"""
from __future__ import annotations


import pytest
import torch
import torch.multiprocessing as mp

from fp4_attn_b200 import shard
from oracle import torch_port as tp


def test_balanced_range_covers_once():
    for n in (0, 1, 7, 8, 33, 1000):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                s, e = shard.balanced_range(n, world, r)
                assert 0 <= s <= e <= n
                seen.extend(range(s, e))
            assert seen == list(range(n))
            sizes = [shard.balanced_range(n, world, r)[1] - shard.balanced_range(n, world, r)[0] for r in range(world)]
            assert max(sizes) - min(sizes) <= 1


def test_bad_arguments():
    with pytest.raises(ValueError):
        shard.balanced_range(4, 2, 2)
    with pytest.raises(ValueError):
        shard.attention_units(1, 6, 4)


def test_attention_units_partition():
    B, Hq, Hkv = 4, 64, 8  # the long-context prefill shape: 32 units
    all_units = set()
    for world in (1, 2, 4, 8):
        got = []
        for r in range(world):
            got += shard.attention_shard(B, Hq, Hkv, world, r)
        assert len(got) == B * Hkv and len(set(got)) == B * Hkv
        all_units |= set(got)
    assert all_units == set(shard.attention_units(B, Hq, Hkv))


def _rendezvous(tmp_path):
    """A file store per test: no TCP port to pick, so no race with other processes for one."""
    return "file://" + str(tmp_path / "rendezvous")


def _attention_rank(rank, world, init, q, k, v, ret):
    torch.distributed.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        B, Hq, T, D = q.shape
        Hkv = k.shape[1]
        Qf, Kf, Vf = tp.fake_quant_qkv(q, k, v)  # whole [B*T, H*D] views, as the reference does
        parts = {}
        for u in shard.attention_shard(B, Hq, Hkv, world, rank):
            qu, ku, vu = shard.unit_inputs(Qf, Kf, Vf, u)
            o = tp.eager_attention(qu, ku, vu, causal=True, scaling=D ** -0.5)  # [1, T, G, D]
            parts[(u.b, u.hk)] = o[0]
        gathered = shard.gather_to_rank0(parts)
        if rank == 0:
            merged = {}
            for p in gathered:
                assert not (set(p) & set(merged)), "a unit was computed twice"
                merged.update(p)
            ret.put(shard.assemble_attention(merged, B, T, Hq, Hkv, D))
    finally:
        torch.distributed.destroy_process_group()


def test_attention_sharded_equals_unsharded(tmp_path):
    g = torch.Generator().manual_seed(7)
    B, Hq, Hkv, T, D = 2, 8, 2, 64, 32
    q = torch.randn(B, Hq, T, D, generator=g).bfloat16()
    k = torch.randn(B, Hkv, T, D, generator=g).bfloat16()
    v = torch.randn(B, Hkv, T, D, generator=g).bfloat16()
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    init = _rendezvous(tmp_path)
    procs = [ctx.Process(target=_attention_rank, args=(r, 2, init, q, k, v, ret)) for r in range(2)]
    for p in procs:
        p.start()
    out = ret.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = tp.attention(q, k, v, causal=True)
    assert torch.equal(out, ref)


def _quant_rank(rank, world, init, x, ret):
    torch.distributed.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        rows = shard.row_shard(x.shape[0], world, rank)
        xs = x[rows].float()
        amax = shard.tensor_amax(xs.abs().amax() if xs.numel() else torch.tensor(0.0))
        one = torch.tensor(1.0)
        gscale = amax * (one / torch.tensor(2688.0))
        y = tp.fused_qdq(xs * (one / gscale), aligned=True, global_sf_max=None) * gscale
        gathered = shard.gather_to_rank0((rows.start, rows.stop, y, amax))
        if rank == 0:
            ret.put(gathered)
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("plant_nan", [False, True])
def test_tensor_mode_row_shards(plant_nan, tmp_path):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(37, 48, generator=g)
    x[5, 7] *= 40.0  # the tensor max lives on rank 0's rows
    if plant_nan:
        x[30, 2] = float("nan")  # and a NaN on rank 1's rows
    x = x.bfloat16()
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    init = _rendezvous(tmp_path)
    procs = [ctx.Process(target=_quant_rank, args=(r, 2, init, x, ret)) for r in range(2)]
    for p in procs:
        p.start()
    parts = ret.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    xf = x.float()
    amax = xf.abs().amax()
    for _, _, _, a in parts:
        assert torch.equal(a.isnan(), amax.reshape(1).isnan())
        if not plant_nan:
            assert torch.equal(a, amax.reshape(1))
    one = torch.tensor(1.0)
    gscale = amax * (one / torch.tensor(2688.0))
    ref = tp.fused_qdq(xf * (one / gscale), aligned=True, global_sf_max=None) * gscale
    got = torch.cat([y for _, _, y, _ in sorted(parts, key=lambda t: t[0])])
    assert got.shape == ref.shape
    assert torch.equal(got.isnan(), ref.isnan())
    assert torch.equal(torch.nan_to_num(got), torch.nan_to_num(ref))
