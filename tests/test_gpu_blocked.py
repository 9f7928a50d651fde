"""Generalised (fanout, leaf block) mode on the GPU against its CPU restatement
(oracle/blocked_oracle.py; parity with the reference is unpinned for this mode -- it has no
counterpart there -- except through the f=2, Lb=1 reduction tested on CPU)."""

import numpy as np
import pytest
import torch

from oracle import blocked_oracle as BO
from tests.tolerance import assert_within
from treeattn_b200 import _lib as L
from treeattn_b200 import blocked as TB
from treeattn_b200.sharding import shard_for_rank

pytestmark = pytest.mark.gpu
DEV = "cuda"
DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}

CASES = [  # (B, N, H, D, S, fanout, leaf_block)
    (1, 256, 2, 64, 4, 2, 16),
    (2, 512, 2, 32, 8, 4, 32),
    (1, 128, 3, 128, 4, 8, 2),
    (1, 64, 2, 64, 3, 2, 1),
    (1, 1024, 1, 96, 8, 4, 64),
]


def _inputs(B, N, H, D, dtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return [torch.randn(B, N, H, D, device=DEV, generator=g).to(DT[dtype]) for _ in range(4)]


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("case", CASES)
def test_forward_backward_against_oracle(case, causal):
    B, N, H, D, S, f, Lb = case
    q, k, v, go = _inputs(B, N, H, D, "f32", N + f)
    dp = BO.depth_of(N, f, Lb)
    rng = np.random.default_rng(N)
    g = rng.gumbel(size=(dp, N, B, H, S, f)).astype(np.float32)
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    out, blk, w = TB.blocked_tree_attention(qq, kk, vv, causal, None, num_samples=S, fanout=f,
                                            leaf_block=Lb, gumbels=torch.from_numpy(g),
                                            return_paths=True)
    out.backward(go)
    sb = lambda t: t.detach().transpose(0, 1).float().cpu().numpy()  # noqa: E731 (seq, B, H, D)
    res = BO.forward(sb(q), sb(k), sb(v), g, S, f, Lb, causal=causal)
    np.testing.assert_array_equal(blk.cpu().numpy(), res["block"])
    np.testing.assert_allclose(w.cpu().numpy(), res["weights"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(sb(out), res["out"], rtol=1e-4, atol=1e-5)
    t64 = lambda x: torch.tensor(sb(x), dtype=torch.float64, requires_grad=True)  # noqa: E731
    q64, k64, v64 = t64(q), t64(k), t64(v)
    ref = BO.forward_torch(q64, k64, v64, res["block"], f, Lb, causal=causal)
    ref.backward(torch.tensor(sb(go), dtype=torch.float64))
    for name, mine, want in (("dq", qq.grad, q64.grad), ("dk", kk.grad, k64.grad), ("dv", vv.grad, v64.grad)):
        np.testing.assert_allclose(sb(mine), want.numpy(), rtol=2e-4, atol=2e-4, err_msg=name)


@pytest.mark.parametrize("dtype,tol", [("bf16", 2e-2), ("f16", 5e-3)])
@pytest.mark.parametrize("N,D,f,Lb", [
    (1024, 128, 4, 64),    # tensor-core forward and backward
    (512, 64, 2, 16),      # tensor-core forward, CUDA-core backward (leaf block 16)
    (2048, 128, 2, 32),
    (1024, 64, 2, 64),
    (2048, 64, 4, 128),
    (2048, 128, 2, 128),   # tensor-core forward, CUDA-core backward (Lb * D > 8192)
    (256, 96, 2, 32),      # head_dim 96: CUDA cores throughout
])
def test_low_precision_within_tolerance(dtype, tol, N, D, f, Lb):
    B, H, S = 2, 2, 8
    q, k, v, go = _inputs(B, N, H, D, dtype, 3)
    if dtype == "f16":
        q, k, v, go = (t * 0.5 for t in (q, k, v, go))
    rng = np.random.default_rng(1)
    g = rng.gumbel(size=(BO.depth_of(N, f, Lb), N, B, H, S, f)).astype(np.float32)
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    out, blk, _ = TB.blocked_tree_attention(qq, kk, vv, True, None, num_samples=S, fanout=f,
                                            leaf_block=Lb, gumbels=torch.from_numpy(g), return_paths=True)
    out.backward(go)
    sb = lambda t: t.detach().transpose(0, 1).double().cpu()  # noqa: E731
    q64, k64, v64 = (sb(t).requires_grad_(True) for t in (q, k, v))
    ref = BO.forward_torch(q64, k64, v64, blk.cpu().numpy(), f, Lb, causal=True)
    ref.backward(sb(go))
    assert_within(sb(out).numpy(), ref.detach().numpy(), dtype, "out", atol=tol)
    for name, mine, want in (("dq", qq.grad, q64.grad), ("dk", kk.grad, k64.grad), ("dv", vv.grad, v64.grad)):
        assert_within(sb(mine).numpy(), want.numpy(), dtype, name, atol=tol)


def test_in_kernel_noise_equals_dumped_noise_and_backward_is_deterministic():
    B, N, H, D, S, f, Lb = 1, 2048, 4, 64, 8, 2, 32
    q, k, v, go = _inputs(B, N, H, D, "bf16", 9)
    torch.manual_seed(123)
    out1, blk1, _ = TB.blocked_tree_attention(q, k, v, False, None, num_samples=S, fanout=f,
                                              leaf_block=Lb, return_paths=True)
    torch.manual_seed(123)
    gen = torch.cuda.default_generators[0]
    cfg = L.Blocked(f, Lb, 0, D ** -0.5, 0, N, 0, B, 0, H)
    shape = L.Shape(B, N, N, H, D, S, L.TA_BF16, 1e3)
    rng = L.Rng(gen.initial_seed(), gen.get_offset(), 0, 1)
    g = TB.gumbel_fill(shape, cfg, rng, DEV)
    out2, blk2, _ = TB.blocked_tree_attention(q, k, v, False, None, num_samples=S, fanout=f,
                                              leaf_block=Lb, gumbels=g, return_paths=True)
    assert torch.equal(blk1, blk2) and torch.equal(out1, out2)
    assert torch.isfinite(g).all() and g.std() > 0.5
    grads = []
    for _ in range(2):
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        TB.blocked_tree_attention(qq, kk, vv, False, None, num_samples=S, fanout=f, leaf_block=Lb,
                                  gumbels=g).backward(go)
        grads.append((qq.grad, kk.grad, vv.grad))
    for a, b in zip(*grads):
        assert torch.equal(a, b)


@pytest.mark.parametrize("axis", ["head", "batch"])
def test_shards_equal_slices_of_the_full_call(axis):
    B, N, H, D, S, f, Lb = 2, 512, 4, 64, 8, 4, 8
    q, k, v, go = _inputs(B, N, H, D, "bf16", 5)

    def run(qq, kk, vv, gg, shard):
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (qq, kk, vv))
        torch.manual_seed(99)
        out = TB.blocked_tree_attention(qq, kk, vv, True, None, num_samples=S, fanout=f,
                                        leaf_block=Lb, shard=shard)
        out.backward(gg)
        return out.detach(), qq.grad, kk.grad, vv.grad

    full = run(q, k, v, go, None)
    for r in range(2):
        spec = shard_for_rank(B, H, r, 2, axis)
        bs, hs = spec.slices()
        part = run(*(t[bs, :, hs].contiguous() for t in (q, k, v, go)), spec)
        for a, b_ in zip(part, full):
            assert torch.equal(a, b_[bs, :, hs])


def test_rejects_bad_geometry():
    x = torch.zeros(1, 96, 1, 32, device=DEV)
    with pytest.raises(ValueError):
        TB.blocked_tree_attention(x, x, x, num_samples=2, fanout=2, leaf_block=64)
    with pytest.raises(ValueError):
        TB.blocked_tree_attention(x[:, :64], x[:, :64], x[:, :64], num_samples=2, fanout=3, leaf_block=1)
