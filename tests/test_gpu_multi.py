"""Multi-GPU (NCCL, one process per GPU): head/batch shards and sequence-parallel chunks
equal their slice of the unsharded call, which every rank also computes on its own GPU.
Skipped with fewer than two GPUs. No kernel waits on another rank; the only cross-GPU
traffic is NCCL all-gather / reduce-scatter (NVLS off)."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(B, N, H, D, dtype, dev):
    gen = torch.Generator(device=dev).manual_seed(21)
    return [torch.randn(B, N, H, D, device=dev, generator=gen).to(dtype) for _ in range(4)]


def _reference(q, k, v, go, S, causal):
    import treeattn_b200 as ta
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    torch.manual_seed(99)
    out = ta.tree_attention(qq, kk, vv, causal, None, num_samples=S)
    out.backward(go)
    return out.detach(), qq.grad, kk.grad, vv.grad


def _worker(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    import treeattn_b200 as ta
    from treeattn_b200.sequence_parallel import sp_tree_attention
    from treeattn_b200.sharding import shard_for_rank

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev)
    msgs = []
    try:
        # head sharding: no collective
        B, N, H, D, S = 1, 1024, 8, 64, 8
        q_, k_, v_, go = _inputs(B, N, H, D, torch.bfloat16, dev)
        ref = _reference(q_, k_, v_, go, S, False)
        spec = shard_for_rank(B, H, rank, WORLD, "head")
        bs, hs = spec.slices()
        qq, kk, vv = (t[bs, :, hs].contiguous().requires_grad_(True) for t in (q_, k_, v_))
        torch.manual_seed(99)
        out = ta.tree_attention(qq, kk, vv, False, None, num_samples=S, shard=spec)
        out.backward(go[bs, :, hs].contiguous())
        for name, a, b in zip(("out", "dq", "dk", "dv"), (out.detach(), qq.grad, kk.grad, vv.grad), ref):
            if not torch.equal(a, b[bs, :, hs]):
                msgs.append(f"shard {name}")
        # sequence parallel, causal and not
        for causal in (False, True):
            B, N, H, D, S = 1, 2048, 4, 128, 16
            q_, k_, v_, go = _inputs(B, N, H, D, torch.bfloat16, dev)
            ref = _reference(q_, k_, v_, go, S, causal)
            n = N // WORLD
            sl = slice(rank * n, (rank + 1) * n)
            qq, kk, vv = (t[:, sl].contiguous().requires_grad_(True) for t in (q_, k_, v_))
            torch.manual_seed(99)
            out = sp_tree_attention(qq, kk, vv, causal, num_samples=S)
            out.backward(go[:, sl].contiguous())
            # sampled rows bit for bit; the exact causal prefix (the first S positions, split
            # over the ranks by heads) up to its split-K summation order
            got, want = out.detach(), ref[0][:, sl]
            e = max(0, min(S, N) - rank * n) if causal and N > S else 0
            if not torch.equal(got[:, e:], want[:, e:]):
                msgs.append(f"sp causal={causal} out")
            if e and not torch.allclose(got[:, :e].float(), want[:, :e].float(), rtol=8e-3, atol=2e-3):
                msgs.append(f"sp causal={causal} prefix out")
            for name, a, b in zip(("dq", "dk", "dv"), (qq.grad, kk.grad, vv.grad), ref[1:]):
                if not torch.allclose(a.float(), b[:, sl].float(), rtol=2e-2, atol=2e-2):
                    msgs.append(f"sp causal={causal} {name}")
        torch.cuda.synchronize()
        q.put((rank, msgs))
    except BaseException as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, [repr(e)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_two_gpus_nccl():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert all(not m for _, m in res), res
