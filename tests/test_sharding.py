"""Host logic of head/batch sharding: partitions, shard specs, and the multi-process
plumbing (gloo, world_size 2, on CPU)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from treeattn_b200.sharding import (ShardSpec, gather_heads, max_over_ranks, partition,
                                    shard_for_rank)


@pytest.mark.parametrize("total,world", [(16, 1), (16, 2), (16, 8), (32, 8), (7, 3), (9, 4), (8, 8)])
def test_partition_is_a_contiguous_cover(total, world):
    covered = []
    for r in range(world):
        start, count = partition(total, r, world)
        assert count >= 1
        covered.extend(range(start, start + count))
    assert covered == list(range(total))
    sizes = [partition(total, r, world)[1] for r in range(world)]
    assert max(sizes) - min(sizes) <= 1


def test_partition_rejects_bad_worlds():
    with pytest.raises(ValueError):
        partition(4, 0, 8)
    with pytest.raises(ValueError):
        partition(4, 3, 2)
    with pytest.raises(ValueError):
        partition(4, 0, 0)


@pytest.mark.parametrize("B,H,world,axis", [(8, 32, 8, "auto"), (1, 16, 4, "auto"), (4, 16, 2, "head"),
                                             (8, 32, 2, "batch"), (1, 32, 8, "head")])
def test_shards_cover_every_unit_once(B, H, world, axis):
    seen = []
    for r in range(world):
        spec = shard_for_rank(B, H, r, world, axis)
        assert spec.batch_total == B and spec.head_total == H
        seen.extend(spec.units())
    assert sorted(seen) == [(b, h) for b in range(B) for h in range(H)]
    assert len(seen) == B * H


def test_shard_spec_validation():
    ShardSpec(2, 0, 2, 4, 0, 4)
    assert ShardSpec(2, 0, 2, 4, 0, 4).is_full
    assert not ShardSpec(2, 1, 1, 4, 0, 4).is_full
    for bad in [(2, 1, 2, 4, 0, 4), (2, 0, 0, 4, 0, 4), (2, 0, 2, 4, 3, 2), (0, 0, 1, 4, 0, 4),
                (2, -1, 1, 4, 0, 4)]:
        with pytest.raises(ValueError):
            ShardSpec(*bad)


def test_bshd_op_refuses_causal_shards():
    from treeattn_b200 import tree_attention
    x = torch.zeros(1, 8, 2, 16)
    with pytest.raises(ValueError, match="causal"):
        tree_attention(x, x, x, True, None, num_samples=2, shard=ShardSpec(1, 0, 1, 4, 0, 2))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, axis, B, H, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        spec = shard_for_rank(B, H, rank, world, axis)
        # every rank's units, gathered: a disjoint cover of the (batch, head) grid
        units = [None] * world
        dist.all_gather_object(units, spec.units())
        flat = [u for part in units for u in part]
        ok_cover = sorted(flat) == [(b, h) for b in range(B) for h in range(H)] and len(flat) == B * H
        # the timing rule: max over ranks
        ok_max = max_over_ranks(float(rank + 1)) == float(world)
        # a per-rank computation on the shard only, gathered back = the full computation
        bs, hs = spec.slices()
        full = torch.arange(B * 4 * H * 2, dtype=torch.float32).view(B, 4, H, 2)
        local = full[bs, :, hs] * 2.0 + 1.0
        ok_gather = torch.equal(gather_heads(local, spec), full * 2.0 + 1.0)
        q.put((rank, ok_cover, ok_max, ok_gather))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("axis,B,H", [("head", 1, 4), ("batch", 2, 3)])
def test_gloo_two_ranks(axis, B, H):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, axis, B, H, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(all(r[1:]) for r in results), results
