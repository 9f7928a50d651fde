"""Parity at the benchmarked configurations (C3 and the headline C5 point).

* Headline (reference semantics): B=1, S=16384, d=128, 8 paths per query, the full Haar tree
  build, noise from torch's CUDA generator exactly as the reference draws it
  (_autograd.py:188-195), through the public bshd op. Two of the sixteen heads (the heads are
  independent trees; two keep the CPU oracle to seconds). Sampled leaves are bit-exact with
  the oracle except classified near ties; out and dq/dk/dv are checked along the sampled
  paths at the north-star bar (max-abs 2e-2 bf16 / 5e-3 fp16, plus at most 2 ulps of the
  output dtype at |ref|, ``tests/tolerance.py``).
* C2 / C3 (generalised fanout / leaf-block mode, no reference counterpart, checked against
  its CPU restatement ``oracle/blocked_oracle.py``): sampled leaf blocks under injected noise
  against the restatement's own sampling, out and gradients along those blocks, at the
  configurations' sizes for a subset of heads.
"""

import numpy as np
import pytest
import torch

import treeattn_b200 as ta
from oracle import blocked_oracle as BO
from oracle import tree_oracle as O
from tests.test_gpu_parity import assert_leaves_match, reference_gumbels
from tests.tolerance import assert_within
from treeattn_b200 import blocked as TB
from treeattn_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"
TDT = {"bf16": torch.bfloat16, "f16": torch.float16}


def _inputs(B, S, H, D, dtype, sigma, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return [(torch.randn(B, S, H, D, device=DEV, generator=g) * sigma).to(TDT[dtype]) for _ in range(4)]


f32 = lambda t: t.detach().float().cpu().numpy()  # noqa: E731


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_headline_shape_against_oracle(dtype):
    B, S, H, D, P = 1, 16384, 2, 128, 8
    q, k, v, go = _inputs(B, S, H, D, dtype, 1.0, 0)
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    torch.manual_seed(11)
    out = ta.tree_attention(qq, kk, vv, False, None, num_samples=P)
    out.backward(go)
    # the same call at op level, for its sampled leaves (same seed: same draws)
    torch.manual_seed(11)
    k_int = ops.tree_build(k.transpose(0, 1))
    res = ops.forward(q.transpose(0, 1), k_int, v.transpose(0, 1), P)
    assert torch.equal(res.out, out.detach().transpose(0, 1))
    torch.manual_seed(11)
    g = reference_gumbels((S, B, H, P, 2), O.log_n_of(S)).cpu().numpy()
    leaf = res.leaf.cpu().numpy().astype(np.int64)

    qs = np.transpose(f32(q), (1, 0, 2, 3))
    k_ref = O.haar_internal_node_keys(np.transpose(f32(k), (1, 0, 2, 3)), dtype)
    np.testing.assert_array_equal(f32(k_int), k_ref)  # tree build bit-exact
    want_leaf, _, _ = O.sample_paths(qs, k_ref, g, P)
    assert_leaves_match(leaf, want_leaf, qs, k_ref, g)

    ref = O.adapter_forward_backward_given_leaves(f32(q), f32(k), f32(v), f32(go), leaf, dtype)
    assert_within(f32(out), ref["out"], dtype, "out")
    for name, t in (("dq", qq), ("dk", kk), ("dv", vv)):
        assert_within(f32(t.grad), ref[name], dtype, name)


def _blocked_ties(q, summ, g, blk_got, blk_want, f, causal, N, rel=2e-6):
    """Every mismatching block must come from a near-tie decision on the restatement's path."""
    bad = np.argwhere(blk_got != blk_want)
    L = q.shape[0]
    dp = len(summ)
    for (l, b, h, s) in bad:
        j, tie = 0, False
        for d in range(dp):
            idx = j * f + np.arange(f)
            z = summ[d][idx, b, h] @ q[l, b, h]
            valid = np.ones(f, bool)
            if causal:
                span = N // f ** (d + 1)
                valid = idx * span <= l + N - L
            zz = np.where(valid, z, -np.inf)
            lsm = zz - zz.max() - np.log(np.exp(zz - zz.max()).sum())
            sc = np.sort(np.where(valid, lsm + g[d, l, b, h, s], -np.inf))[::-1]
            if valid.sum() > 1 and sc[0] - sc[1] < rel * max(1.0, abs(sc[0])):
                tie = True
                break
            j = j * f + int((blk_want[l, b, h, s] // f ** (dp - d - 1)) % f)
        assert tie, f"leaf-block mismatch at {(l, b, h, s)} that is not a near tie"
    assert len(bad) <= max(2, blk_got.size // 10000), f"too many near-tie mismatches: {len(bad)}"
    return bad


# C2: B=4, S=4096, H=16 (1 of 16 here), d=128 bf16 N(0,1), f=2, Lb=64, 8 paths, non-causal.
# C3: B=8 (1 here), S=8192, H=32 (2 here), d=64 fp16 N(0,0.5), f=4, Lb=128, 8 paths, causal.
@pytest.mark.parametrize("name,B,S,H,D,dtype,sigma,f,Lb,causal", [
    ("C2", 4, 4096, 1, 128, "bf16", 1.0, 2, 64, False),
    ("C3", 1, 8192, 2, 64, "f16", 0.5, 4, 128, True),
])
def test_blocked_configs_against_restatement(name, B, S, H, D, dtype, sigma, f, Lb, causal):
    P = 8
    q, k, v, go = _inputs(B, S, H, D, dtype, sigma, 1)
    dp = BO.depth_of(S, f, Lb)
    g = np.random.default_rng(5).gumbel(size=(dp, S, B, H, P, f)).astype(np.float32)
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    out, blk, _ = TB.blocked_tree_attention(qq, kk, vv, causal, None, num_samples=P, fanout=f,
                                            leaf_block=Lb, gumbels=torch.from_numpy(g),
                                            return_paths=True)
    out.backward(go)
    blk = blk.cpu().numpy().astype(np.int64)
    sb = lambda t: np.ascontiguousarray(np.transpose(f32(t), (1, 0, 2, 3)))  # noqa: E731
    qs, ks, vs, gos = sb(q), sb(k), sb(v), sb(go)
    summ = BO.summaries(ks, f, Lb)

    # sampled blocks: the restatement's own sampling under the same noise
    want = np.empty_like(blk)
    chunk = 1024
    for a in range(0, S, chunk):
        want[a:a + chunk], _ = BO.sample_blocks(qs[a:a + chunk], summ, g[:, a:a + chunk], P, f, Lb, S,
                                                causal, query_start=a, total_queries=S)
    _blocked_ties(qs, summ, g, blk, want, f, causal, S)

    # values along the GPU's blocks: float32 torch autograd of the restatement, a query slice
    # at a time (dK / dV accumulate over the slices)
    kt = torch.tensor(ks, requires_grad=True)
    vt = torch.tensor(vs, requires_grad=True)
    out_ref = np.empty_like(qs)
    dq_ref = np.empty_like(qs)
    chunk = 256
    for a in range(0, S, chunk):
        qt = torch.tensor(qs[a:a + chunk], requires_grad=True)
        o = BO.forward_torch(qt, kt, vt, blk[a:a + chunk], f, Lb, causal=causal, query_start=a,
                             total_queries=S)
        o.backward(torch.from_numpy(gos[a:a + chunk]))
        out_ref[a:a + chunk] = o.detach().numpy()
        dq_ref[a:a + chunk] = qt.grad.numpy()
    assert_within(sb(out), out_ref, dtype, f"{name} out")
    assert_within(sb(qq.grad), dq_ref, dtype, f"{name} dq")
    assert_within(sb(kk.grad), kt.grad.numpy(), dtype, f"{name} dk")
    assert_within(sb(vv.grad), vt.grad.numpy(), dtype, f"{name} dv")
