"""GPU parity: the CUDA path against the oracle and the reference's golden fixtures.

Mirrors the reference's own tests (packages/attn-bench/tests/test_harness_smoke.py):
sampler bit-equality under a fixed seed (:325-421), replay round trip (:110-211), backward
pieces (:214-821) and the end-to-end comparison at five shapes with the same tolerances
(:824-917). The oracle is tests-only (oracle/tree_oracle.py); every call under test goes
through the C ABI of libtreeattn_b200.so.
"""

import glob
import os

import numpy as np
import pytest
import torch

import treeattn_b200 as ta
from oracle import tree_oracle as O
from tests.conftest import GOLDEN
from tests.tolerance import assert_within
from treeattn_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"
ATTN = sorted(glob.glob(os.path.join(GOLDEN, "attn_*.npz")))
ADAPTER = sorted(glob.glob(os.path.join(GOLDEN, "adapter_*.npz")))
HAAR = sorted(glob.glob(os.path.join(GOLDEN, "haar_*.npz")))
TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def _t(x, dt=torch.float32):
    return torch.as_tensor(np.asarray(x)).to(device=DEV, dtype=dt)


def reference_gumbels(shape, log_n):
    """The reference's per-depth draw (_autograd.py:188-195) from torch's CUDA generator."""
    return torch.stack([torch.empty(shape, device=DEV, dtype=torch.float32).exponential_().log_().neg_()
                        for _ in range(log_n)])


def assert_leaves_match(got, want, q, k, gumbels, tol=2e-6):
    """Leaves must be identical, except where the oracle's decision was a near tie."""
    got = np.asarray(got)
    want = np.asarray(want)
    bad = np.argwhere(got != want)
    if len(bad) == 0:
        return
    # classify each mismatch: replay the oracle path and look for a near-tie decision
    q32, k32 = np.asarray(q, np.float32), np.asarray(k, np.float32)
    log_n = gumbels.shape[0]
    K = k32.shape[0]
    for (l, b, h, s) in bad:
        node, tie = 0, False
        for d in range(log_n):
            x = np.clip(np.float32(q32[l, b, h] @ k32[node, b, h]), -1e3, 1e3)
            lp_l, lp_r = O.log_sigmoid_pair(np.array([x], np.float32))
            margin = abs(float(lp_r[0] + gumbels[d, l, b, h, s, 1]) - float(lp_l[0] + gumbels[d, l, b, h, s, 0]))
            if margin < tol * max(1.0, abs(float(lp_l[0]) + float(gumbels[d, l, b, h, s, 0]))):
                tie = True
                break
            node = 2 * node + 1 + int(((want[l, b, h, s] + K + 1) >> (log_n - 1 - d)) & 1)
        assert tie, f"leaf mismatch at {(l, b, h, s)} that is not a near tie"
    assert len(bad) <= max(2, got.size // 10000), f"too many near-tie mismatches: {len(bad)}"


# ---------------------------------------------------------------------------------------
# Gumbel stream
# ---------------------------------------------------------------------------------------

@pytest.mark.parametrize("numel", [8, 1000, 4096 * 2, 303104, 303104 + 6, 1_234_566, 4 * 1024 * 1024])
def test_gumbel_stream_bit_exact_with_torch(numel):
    torch.manual_seed(123)
    rng = ops.reserve_gumbel_stream(torch.device(DEV), numel, 3)
    after = torch.cuda.default_generators[0].get_offset()
    torch.manual_seed(123)
    ref = reference_gumbels((numel,), 3)
    assert torch.cuda.default_generators[0].get_offset() == after  # same offsets consumed
    for d in range(3):
        got = ops.gumbel_fill(torch.empty(numel, device=DEV), rng, d)
        assert torch.equal(got, ref[d]), f"depth {d}: {(got != ref[d]).sum().item()} differ"
    allg = ops.gumbel_fill(torch.empty(3, numel, device=DEV), rng)
    assert torch.equal(allg, ref)


# ---------------------------------------------------------------------------------------
# sampler / replay (test_harness_smoke.py:110-211, 325-421)
# ---------------------------------------------------------------------------------------

@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("L,B,H,D,S", [(8, 1, 2, 16, 4), (32, 2, 2, 16, 4), (256, 1, 4, 64, 8),
                                       (512, 2, 4, 32, 8), (64, 1, 2, 128, 5), (128, 1, 3, 96, 16)])
def test_sampler_matches_oracle_and_reference_stream(dtype, L, B, H, D, S):
    dt = TORCH_DT[dtype]
    if dt != torch.float32 and D * 2 % 16:
        pytest.skip("row not 16-byte aligned")
    torch.manual_seed(0)
    q = torch.randn(L, B, H, D, device=DEV).to(dt)
    k = torch.randn(L - 1, B, H, D, device=DEV).to(dt)
    log_n = O.log_n_of(L)
    torch.manual_seed(123)
    leaf, lp, packed = ops.sample_paths(q, k, S)
    torch.manual_seed(123)
    g = reference_gumbels((L, B, H, S, 2), log_n)
    qn, kn, gn = q.float().cpu().numpy(), k.float().cpu().numpy(), g.cpu().numpy()
    want_leaf, want_lp, want_packed = O.sample_paths(qn, kn, gn, S)
    assert_leaves_match(leaf.cpu().numpy(), want_leaf, qn, kn, gn)
    same = leaf.cpu().numpy() == want_leaf
    np.testing.assert_allclose(lp.cpu().numpy()[same], want_lp[same], rtol=1e-5, atol=1e-5)
    # injected noise gives the identical result
    leaf2, lp2, packed2 = ops.sample_paths(q, k, S, gumbels=g)
    assert torch.equal(leaf2, leaf) and torch.equal(packed2, packed) and torch.equal(lp2, lp)
    # replay round trip
    rl, rlp = ops.replay_paths(q, k, packed)
    assert torch.equal(rl, leaf)
    torch.testing.assert_close(rlp, lp, rtol=0, atol=0)
    rl2, rw = ops.replay_paths(q, k, packed, softmax=True)
    torch.testing.assert_close(rw, torch.softmax(lp, dim=-1), rtol=1e-5, atol=1e-6)
    assert torch.equal(torch.as_tensor(O.path_bits_from_leaf(leaf.cpu().numpy().astype(np.int64), L)),
                       packed.cpu())


def test_fused_and_prefilled_noise_agree():
    torch.manual_seed(0)
    q = torch.randn(300, 2, 3, 64, device=DEV, dtype=torch.bfloat16)
    k = torch.randn(511, 2, 3, 64, device=DEV, dtype=torch.bfloat16)
    v = torch.randn(512, 2, 3, 64, device=DEV, dtype=torch.bfloat16)
    torch.manual_seed(9)
    a = ops.forward(q, k, v, 8)
    torch.manual_seed(9)
    b = ops.forward(q, k, v, 8, fused_rng=True)
    assert torch.equal(a.leaf, b.leaf) and torch.equal(a.out, b.out)
    assert torch.equal(a.branch_prob, b.branch_prob)


def test_sampler_deterministic_and_seed_sensitive():
    torch.manual_seed(0)
    q = torch.randn(32, 1, 2, 16, device=DEV)
    k = torch.randn(31, 1, 2, 16, device=DEV)
    torch.manual_seed(123)
    a = ops.sample_paths(q, k, 4)
    torch.manual_seed(123)
    b = ops.sample_paths(q, k, 4)
    c = ops.sample_paths(q, k, 4)  # next offsets
    assert torch.equal(a[0], b[0]) and torch.equal(a[2], b[2])
    assert not torch.equal(b[0], c[0])


# ---------------------------------------------------------------------------------------
# golden fixtures from the reference implementation (injected noise)
# ---------------------------------------------------------------------------------------

@pytest.mark.parametrize("path", ATTN, ids=os.path.basename)
def test_forward_backward_match_reference_fixtures(path):
    f = np.load(path)
    L, B, H, D, S = (int(x) for x in f["shape"])
    q = _t(f["q"]).reshape(L, B, H, D)
    k = _t(f["k"]).reshape(L - 1, B, H, D)
    v = _t(f["v"]).reshape(L, B, H, D)
    g = _t(f["grad_out"]).reshape(L, B, H, D)
    res = ops.forward(q, k, v, S, gumbels=_t(f["gumbels"]), want_packed=True)
    np.testing.assert_array_equal(res.leaf.cpu().numpy(), f["leaf"])
    np.testing.assert_array_equal(res.packed.cpu().numpy(), f["cuda_packed"])
    # the reference test's tolerances (test_harness_smoke.py:887-891)
    np.testing.assert_allclose(res.out.reshape(L, B, -1).cpu().numpy(), f["out"], atol=5e-5, rtol=5e-5)
    np.testing.assert_allclose(res.weights.cpu().numpy(), f["weights"], atol=5e-5, rtol=5e-5)
    dq, dk, dv = ops.backward(q, k, v, g, res.leaf, res.weights, res.branch_prob, S)
    np.testing.assert_allclose(dq.reshape(L, B, -1).cpu().numpy(), f["dq"], atol=2e-4, rtol=2e-4)
    np.testing.assert_allclose(dk.reshape(L - 1, B, -1).cpu().numpy(), f["dk"], atol=4e-4, rtol=4e-4)
    np.testing.assert_allclose(dv.reshape(L, B, -1).cpu().numpy(), f["dv"], atol=2e-4, rtol=2e-4)


@pytest.mark.parametrize("path", ADAPTER, ids=os.path.basename)
def test_bshd_adapter_matches_reference_fixtures(path):
    f = np.load(path)
    dt = os.path.basename(path).split("_")[1]
    tdt = TORCH_DT[dt]
    q, k, v, go = (_t(f[n], tdt).requires_grad_(n != "grad_out") for n in ("q", "k", "v", "grad_out"))
    out = ta.tree_attention(q, k, v, False, None, num_samples=int(f["num_samples"]),
                            gumbels=_t(f["gumbels"]))
    out.backward(go)
    tol = {"f32": dict(out=5e-5, g=4e-4), "bf16": dict(out=2e-2, g=5e-2)}[dt]
    np.testing.assert_allclose(out.float().detach().cpu().numpy(), f["out"], atol=tol["out"], rtol=tol["out"])
    for name, t in (("dq", q), ("dk", k), ("dv", v)):
        np.testing.assert_allclose(t.grad.float().cpu().numpy(), f[name], atol=tol["g"],
                                   rtol=tol["g"], err_msg=name)


@pytest.mark.parametrize("path", HAAR, ids=os.path.basename)
def test_tree_build_matches_reference_fixtures(path):
    f = np.load(path)
    dt = TORCH_DT[os.path.basename(path).split("_")[1]]
    k = _t(f["k"], dt)
    if k.shape[-1] * k.element_size() % 16:
        pytest.skip("rows narrower than 16 bytes are not supported by the tree build")
    out = ops.tree_build(k)
    np.testing.assert_array_equal(out.float().cpu().numpy(), f["out"])  # bit-exact
    S, B, H, D = k.shape
    dk = torch.empty_like(k)
    ops.tree_build_backward(_t(f["grad_in"]), dk)
    np.testing.assert_allclose(dk.float().cpu().numpy(), O.haar_internal_node_keys_backward(f["grad_in"]),
                               rtol=1e-2 if dt != torch.float32 else 1e-6, atol=1e-2 if dt != torch.float32 else 1e-6)


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("S", [2, 4, 32, 64, 1024, 2048, 65536])
def test_tree_build_multi_pass_bit_exact(dtype, S):
    dt = TORCH_DT[dtype]
    B, H, D = (1, 2, 16) if S > 4096 else (2, 3, 32)
    torch.manual_seed(S)
    k = torch.randn(B, S, H, D, device=DEV).to(dt)  # bshd
    out = ops.tree_build(k.transpose(0, 1))
    want = O.haar_internal_node_keys(k.transpose(0, 1).float().cpu().numpy(), dtype)
    np.testing.assert_array_equal(out.float().cpu().numpy(), want)
    g = torch.randn(S - 1, B, H, D, device=DEV)
    dk = torch.empty_like(k)
    ops.tree_build_backward(g, dk.transpose(0, 1))
    want_g = O.haar_internal_node_keys_backward(g.cpu().numpy())
    tol = {"f32": 1e-6, "f16": 2e-3, "bf16": 1e-2}[dtype]
    np.testing.assert_allclose(dk.transpose(0, 1).float().cpu().numpy(), want_g, rtol=tol, atol=tol)


# ---------------------------------------------------------------------------------------
# end to end with the generator's noise (test_harness_smoke.py:824-917)
# ---------------------------------------------------------------------------------------

@pytest.mark.parametrize("seqlen,batch,nheads,head_dim,num_samples",
                         [(8, 1, 2, 16, 4), (32, 2, 2, 16, 4), (64, 1, 8, 16, 4), (128, 1, 2, 64, 8),
                          (512, 2, 4, 32, 8)])
def test_hierarchical_attention_matches_reference_semantics(seqlen, batch, nheads, head_dim, num_samples):
    embed = nheads * head_dim
    torch.manual_seed(1234)
    q = torch.randn(seqlen, batch, embed, device=DEV, requires_grad=True)
    k = torch.randn(seqlen - 1, batch, embed, device=DEV, requires_grad=True)
    v = torch.randn(seqlen, batch, embed, device=DEV, requires_grad=True)
    go = torch.randn(seqlen, batch, embed, device=DEV)
    torch.manual_seed(0)
    out, w = ta.hierarchical_attention(q, k, v, num_heads=nheads, num_samples=num_samples,
                                       block_size=min(256, seqlen))
    out.backward(go)
    torch.manual_seed(0)
    g = reference_gumbels((seqlen, batch, nheads, num_samples, 2), O.log_n_of(seqlen)).cpu().numpy()
    qn = q.detach().cpu().numpy().reshape(seqlen, batch, nheads, head_dim)
    kn = k.detach().cpu().numpy().reshape(seqlen - 1, batch, nheads, head_dim)
    vn = v.detach().cpu().numpy().reshape(seqlen, batch, nheads, head_dim)
    fw = O.forward(qn, kn, vn, g, num_samples)
    dq, dk, dv = O.backward(qn, kn, vn, go.cpu().numpy().reshape(qn.shape), fw["leaf"], fw["weights"])
    np.testing.assert_allclose(out.detach().cpu().numpy(), fw["out"].reshape(seqlen, batch, -1), atol=5e-5, rtol=5e-5)
    np.testing.assert_allclose(w.cpu().numpy(), fw["weights"], atol=5e-5, rtol=5e-5)
    np.testing.assert_allclose(q.grad.cpu().numpy(), dq.reshape(seqlen, batch, -1), atol=2e-4, rtol=2e-4)
    np.testing.assert_allclose(k.grad.cpu().numpy(), dk.reshape(seqlen - 1, batch, -1), atol=4e-4, rtol=4e-4)
    np.testing.assert_allclose(v.grad.cpu().numpy(), dv.reshape(seqlen, batch, -1), atol=2e-4, rtol=2e-4)


@pytest.mark.parametrize("dtype,tol", [("bf16", 2e-2), ("f16", 5e-3)])
@pytest.mark.parametrize("B,S,H,D,P", [(2, 256, 4, 64, 8), (1, 1024, 2, 128, 8), (1, 512, 2, 32, 4),
                                       (1, 256, 2, 96, 16)])
def test_low_precision_within_tolerance_of_fp32_oracle(dtype, tol, B, S, H, D, P):
    """north_star tolerance: max-abs 2e-2 (bf16) / 5e-3 (fp16) vs the fp32 reference, plus at
    most 2 ulps of the output dtype at |ref| (tests/tolerance.py), along the sampled paths;
    the sampled leaves themselves equal the oracle's except near ties."""
    dt = TORCH_DT[dtype]
    torch.manual_seed(7)
    scale = 0.5 if dtype == "f16" else 1.0
    q, k, v, go = (torch.randn(B, S, H, D, device=DEV).mul(scale).to(dt) for _ in range(4))
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    torch.manual_seed(3)
    out = ta.tree_attention(qq, kk, vv, num_samples=P)
    out.backward(go)
    torch.manual_seed(3)
    ops_leaf = ops.forward(q.transpose(0, 1), ops.tree_build(k.transpose(0, 1)), v.transpose(0, 1), P).leaf
    ops_leaf = ops_leaf.cpu().numpy()
    torch.manual_seed(3)
    g = reference_gumbels((S, B, H, P, 2), O.log_n_of(S)).cpu().numpy()
    f32 = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
    res_k_int = O.haar_internal_node_keys(np.transpose(f32(k), (1, 0, 2, 3)), dtype)
    res = O.adapter_forward_backward_given_leaves(f32(q), f32(k), f32(v), f32(go), ops_leaf, dtype)
    res["leaf"] = O.sample_paths(np.transpose(f32(q), (1, 0, 2, 3)), res_k_int, g, P)[0]
    assert_leaves_match(ops_leaf, res["leaf"], np.transpose(f32(q), (1, 0, 2, 3)), res_k_int, g)
    assert_within(f32(out), res["out"], dtype, "out", atol=tol)
    for name, t in (("dq", qq), ("dk", kk), ("dv", vv)):
        assert_within(f32(t.grad), res[name], dtype, name, atol=tol)


def test_backward_is_bitwise_deterministic():
    torch.manual_seed(0)
    B, S, H, D = 1, 2048, 4, 128
    q, k, v, go = (torch.randn(B, S, H, D, device=DEV, dtype=torch.bfloat16) for _ in range(4))
    grads = []
    for _ in range(3):
        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        torch.manual_seed(5)
        ta.tree_attention(qq, kk, vv, num_samples=8).backward(go)
        grads.append([t.grad.clone() for t in (qq, kk, vv)])
    for other in grads[1:]:
        for a, b in zip(grads[0], other):
            assert torch.equal(a, b)


def test_edge_shapes_and_layouts():
    """N=2 (one level), one sample, L != N, sbhd and bshd strides, odd sample counts."""
    for (L, N, B, H, D, S) in [(5, 2, 1, 1, 16, 1), (100, 64, 2, 3, 32, 3), (70, 128, 1, 2, 64, 7),
                               (1, 1024, 1, 1, 128, 32)]:
        torch.manual_seed(L + N)
        q = torch.randn(B, L, H, D, device=DEV).transpose(0, 1)  # bshd memory, (L,B,H,D) view
        k = torch.randn(N - 1, B, H, D, device=DEV)
        v = torch.randn(N, B, H, D, device=DEV)
        go = torch.randn(L, B, H, D, device=DEV)
        torch.manual_seed(1)
        g = reference_gumbels((L, B, H, S, 2), O.log_n_of(N))
        res = ops.forward(q, k, v, S, gumbels=g)
        fw = O.forward(*(t.cpu().numpy() for t in (q, k, v, g)), S)
        assert_leaves_match(res.leaf.cpu().numpy(), fw["leaf"], q.cpu().numpy(), k.cpu().numpy(), g.cpu().numpy())
        np.testing.assert_allclose(res.out.cpu().numpy(), fw["out"], atol=5e-5, rtol=5e-5)
        dq, dk, dv = ops.backward(q, k, v, go, res.leaf, res.weights, res.branch_prob, S)
        rq, rk, rv = O.backward(*(t.cpu().numpy() for t in (q, k, v, go)), res.leaf.cpu().numpy().astype(np.int64),
                                res.weights.cpu().numpy())
        np.testing.assert_allclose(dq.cpu().numpy(), rq, atol=2e-4, rtol=2e-4)
        np.testing.assert_allclose(dk.cpu().numpy(), rk, atol=4e-4, rtol=4e-4)
        np.testing.assert_allclose(dv.cpu().numpy(), rv, atol=2e-4, rtol=2e-4)


def test_collapsed_paths_all_queries_one_leaf():
    """Every path ends at the same leaf: one node per level carries all L*S contributions."""
    L, B, H, D, S = 512, 1, 1, 32, 8
    q = torch.ones(L, B, H, D, device=DEV)
    k = torch.full((L - 1, B, H, D), 5.0, device=DEV)  # logit +160: always left
    v = torch.randn(L, B, H, D, device=DEV)
    go = torch.randn(L, B, H, D, device=DEV)
    torch.manual_seed(0)
    res = ops.forward(q, k, v, S)
    assert int(res.leaf.max()) == 0
    dq, dk, dv = ops.backward(q, k, v, go, res.leaf, res.weights, res.branch_prob, S)
    rq, rk, rv = O.backward(*(t.cpu().numpy() for t in (q, k, v, go)), res.leaf.cpu().numpy().astype(np.int64),
                            res.weights.cpu().numpy())
    np.testing.assert_allclose(dv.cpu().numpy(), rv, atol=1e-3, rtol=1e-4)
    np.testing.assert_allclose(dk.cpu().numpy(), rk, atol=1e-3, rtol=1e-4)
    np.testing.assert_allclose(dq.cpu().numpy(), rq, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("L,N,B,H,D,S", [(512, 512, 1, 2, 128, 8), (4, 4096, 1, 1, 64, 8),
                                         (300, 1024, 2, 3, 32, 5), (1024, 256, 1, 2, 96, 16),
                                         (64, 128, 1, 1, 256, 4)])
def test_backward_bf16_tensor_core_node_pass(L, N, B, H, D, S):
    """bf16 head_dim % 32 == 0 takes the mma.sync node pass: dense, sparse (many rows per
    chunk and unreached nodes), odd sample counts, D up to 256."""
    torch.manual_seed(L + N + D)
    q = torch.randn(L, B, H, D, device=DEV, dtype=torch.bfloat16)
    k = torch.randn(N - 1, B, H, D, device=DEV, dtype=torch.bfloat16)
    v = torch.randn(N, B, H, D, device=DEV, dtype=torch.bfloat16)
    go = torch.randn(L, B, H, D, device=DEV, dtype=torch.bfloat16)
    torch.manual_seed(2)
    res = ops.forward(q, k, v, S)
    dq, dk, dv = ops.backward(q, k, v, go, res.leaf, res.weights, res.branch_prob, S,
                              dk_dtype=torch.float32)
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    rq, rk, rv = O.backward(f(q), f(k), f(v), f(go), res.leaf.cpu().numpy().astype(np.int64),
                            res.weights.cpu().numpy())
    np.testing.assert_allclose(f(dk), rk, atol=2e-4, rtol=2e-4)  # float32 output
    np.testing.assert_allclose(f(dv), rv, atol=2e-2, rtol=1e-2)  # bf16 outputs
    np.testing.assert_allclose(f(dq), rq, atol=2e-2, rtol=1e-2)
    # deterministic
    dq2, dk2, dv2 = ops.backward(q, k, v, go, res.leaf, res.weights, res.branch_prob, S,
                                 dk_dtype=torch.float32)
    assert torch.equal(dk, dk2) and torch.equal(dv, dv2) and torch.equal(dq, dq2)


@pytest.mark.parametrize("range_chunks", [1, 3, 32])
@pytest.mark.parametrize("L,N,B,H,D,S", [(2048, 2048, 1, 2, 128, 8), (1000, 64, 2, 1, 64, 3),
                                         (512, 8192, 1, 1, 256, 8)])
def test_node_pass_ranges_carry_open_nodes(range_chunks, L, N, B, H, D, S):
    """The tensor-core node pass walks ranges of 128-path chunks and carries nodes that stay
    open between chunks (deep trees: many nodes span several chunks; shallow trees: every
    node does). Every range size matches the oracle and is bitwise repeatable."""
    from treeattn_b200 import _lib

    lib = _lib.load()
    torch.manual_seed(L + N + D)
    q = torch.randn(L, B, H, D, device=DEV, dtype=torch.bfloat16)
    k = torch.randn(N - 1, B, H, D, device=DEV, dtype=torch.bfloat16)
    v = torch.randn(N, B, H, D, device=DEV, dtype=torch.bfloat16)
    go = torch.randn(L, B, H, D, device=DEV, dtype=torch.bfloat16)
    torch.manual_seed(3)
    res = ops.forward(q, k, v, S)
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    rq, rk, rv = O.backward(f(q), f(k), f(v), f(go), res.leaf.cpu().numpy().astype(np.int64),
                            res.weights.cpu().numpy())
    old = lib.ta_backward_set_node_range(range_chunks)
    try:
        outs = [ops.backward(q, k, v, go, res.leaf, res.weights, res.branch_prob, S,
                             dk_dtype=torch.float32,
                             dv=torch.empty(N, B, H, D, device=DEV, dtype=torch.float32))
                for _ in range(2)]
    finally:
        lib.ta_backward_set_node_range(old)
    dq, dk, dv = outs[0]
    np.testing.assert_allclose(f(dk), rk, atol=2e-4, rtol=2e-4)
    np.testing.assert_allclose(f(dv), rv, atol=2e-4, rtol=2e-4)
    np.testing.assert_allclose(f(dq), rq, atol=2e-2, rtol=1e-2)
    assert all(torch.equal(a, b) for a, b in zip(outs[0], outs[1]))
