"""Sequence parallelism, host side: the query plan and the collectives (gloo, 2 ranks)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from treeattn_b200 import sequence_parallel as sp
from treeattn_b200.sequence_parallel import TorchDistComm, plan, sp_tree_attention


@pytest.mark.parametrize("N,R,S,causal", [(64, 2, 8, True), (64, 4, 16, True), (32, 8, 8, True),
                                          (16, 2, 16, True), (16, 4, 32, True), (64, 4, 8, False)])
def test_plan_covers_queries_in_order(N, R, S, causal):
    sampled_t, exact_q = [], []
    for r in range(R):
        p = plan(N, R, r, S, causal)
        assert p.q0 == r * (N // R) and p.chunk == N // R
        exact_q += list(range(p.q0, p.q0 + p.exact))
        sampled_t += list(range(p.sampled_t0, p.sampled_t0 + p.chunk - p.exact))
        assert p.sampled_offset == p.q0 + p.exact
    if causal and N > S:
        # treeattn-torch: the first S queries exact, the rest sampled from t = 0
        assert exact_q == list(range(min(S, N)))
        assert sampled_t == list(range(N - S))
    else:
        assert exact_q == []
        assert sampled_t == list(range(N))


def test_prefix_balance_rule():
    # the exact prefix (first S queries) splits by heads only inside rank 0's chunk with H % R == 0
    assert plan(64, 2, 0, 8, True).prefix == 8
    assert plan(64, 2, 1, 8, True).balanced(2, 4)
    assert not plan(64, 2, 1, 8, True).balanced(2, 3)
    assert not plan(64, 8, 0, 16, True).balanced(8, 8)   # chunk 8 < prefix 16
    assert not plan(64, 2, 0, 8, False).balanced(2, 4)
    assert not plan(8, 2, 0, 8, True).balanced(2, 4)     # N <= S: no hybrid prefix


def test_plan_rejects_uneven_splits():
    with pytest.raises(ValueError):
        plan(48, 5, 0, 8, True)
    with pytest.raises(ValueError):
        plan(96, 2, 0, 8, True)   # chunk 48 is not a power of two
    with pytest.raises(ValueError):
        plan(64, 2, 2, 8, True)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        comm = TorchDistComm()
        n = 3
        chunk = torch.full((n, 2, 4), float(rank + 1))
        out = torch.empty((n * world, 2, 4))
        comm.all_gather_seq(out, chunk)
        want = torch.cat([torch.full((n, 2, 4), float(r + 1)) for r in range(world)])
        ok_gather = torch.equal(out, want)
        full = torch.arange(n * world * 5, dtype=torch.float32).view(n * world, 5) * (rank + 1)
        mine = torch.empty((n, 5))
        comm.reduce_scatter_seq(mine, full)
        tot = sum(r + 1 for r in range(world))
        ok_rs = torch.equal(mine, torch.arange(n * world * 5, dtype=torch.float32).view(n * world, 5)[rank * n:(rank + 1) * n] * tot)
        # the balanced exact prefix: rank 0's rows reach every rank, head slices come back
        E, B, H, D = 2, 1, 4, 3
        rows = torch.arange(E * B * H * D, dtype=torch.float32).view(E, B, H, D) + 100 * rank
        got = sp._from_rank0(comm, rows)
        ok_bcast = torch.equal(got, rows - 100 * rank)
        hs = sp._prefix_heads(comm, H)
        dst = torch.zeros(E, B, H, D)
        sp._heads_to_rank0(comm, dst, got[:, :, hs].contiguous() * 2)
        ok_heads = (not torch.equal(dst, torch.zeros_like(dst))) if rank == 0 else True
        ok_heads = ok_heads and (rank != 0 or torch.equal(dst, 2 * (rows - 100 * rank)))
        ok_gather = ok_gather and ok_bcast and ok_heads
        # the public entry point validates shapes before any device work
        ok_err = False
        try:
            x = torch.zeros(1, 6, 2, 8)
            sp_tree_attention(x, x, x, True, num_samples=2, comm=comm)
        except ValueError:
            ok_err = True
        q.put((rank, ok_gather, ok_rs, ok_err))
    finally:
        dist.destroy_process_group()


def test_collectives_on_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(all(r[1:]) for r in res), res
