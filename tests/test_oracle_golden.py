"""Pin the numpy oracle against fixtures produced by the reference implementation itself."""

import glob
import os

import numpy as np
import pytest

from oracle import tree_oracle as O
from tests.conftest import GOLDEN

ATTN = sorted(glob.glob(os.path.join(GOLDEN, "attn_*.npz")))
HAAR = sorted(glob.glob(os.path.join(GOLDEN, "haar_*.npz")))
ADAPTER = sorted(glob.glob(os.path.join(GOLDEN, "adapter_*.npz")))


def _heads(x, H):
    return x.reshape(x.shape[0], x.shape[1], H, -1)


def test_fixtures_present():
    assert len(ATTN) == 5 and len(HAAR) == 9 and len(ADAPTER) == 4


@pytest.mark.parametrize("path", ATTN, ids=os.path.basename)
def test_oracle_sampler_matches_reference(path):
    f = np.load(path)
    L, B, H, D, S = (int(x) for x in f["shape"])
    q, k = _heads(f["q"], H), _heads(f["k"], H)
    leaf, lp, packed = O.sample_paths(q, k, f["gumbels"], S)
    # treeattn-torch and treeattn-cuda (python path) agree with each other ...
    np.testing.assert_array_equal(f["leaf"], f["cuda_leaf"])
    # ... and the oracle reproduces the reference's sampled leaves and packed bits exactly
    np.testing.assert_array_equal(leaf, f["leaf"])
    np.testing.assert_array_equal(packed, f["cuda_packed"])
    np.testing.assert_allclose(lp, f["log_prob"], rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(O.path_bits_from_leaf(leaf, L), packed)
    rl, rlp = O.replay_paths(q, k, packed)
    np.testing.assert_array_equal(rl, leaf)
    np.testing.assert_allclose(rlp, lp, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("path", ATTN, ids=os.path.basename)
def test_oracle_forward_backward_matches_reference(path):
    f = np.load(path)
    L, B, H, D, S = (int(x) for x in f["shape"])
    q, k, v, g = (_heads(f[n], H) for n in ("q", "k", "v", "grad_out"))
    fw = O.forward(q, k, v, f["gumbels"], S)
    # the reference test's own tolerances (test_harness_smoke.py:887-891)
    for tag in ("", "cuda_"):
        np.testing.assert_allclose(fw["out"].reshape(L, B, -1), f[tag + "out"], atol=5e-5, rtol=5e-5)
        np.testing.assert_allclose(fw["weights"], f[tag + "weights"], atol=5e-5, rtol=5e-5)
    dq, dk, dv = O.backward(q, k, v, g, fw["leaf"], fw["weights"])
    for tag in ("", "cuda_"):
        np.testing.assert_allclose(dq.reshape(L, B, -1), f[tag + "dq"], atol=2e-4, rtol=2e-4)
        np.testing.assert_allclose(dk.reshape(L - 1, B, -1), f[tag + "dk"], atol=4e-4, rtol=4e-4)
        np.testing.assert_allclose(dv.reshape(L, B, -1), f[tag + "dv"], atol=2e-4, rtol=2e-4)


@pytest.mark.parametrize("path", HAAR, ids=os.path.basename)
def test_oracle_haar_matches_reference(path):
    f = np.load(path)
    dt = os.path.basename(path).split("_")[1]
    out = O.haar_internal_node_keys(f["k"], dt)
    np.testing.assert_array_equal(out, f["out"])  # bit-exact, op-by-op dtype rounding
    gk = O.haar_internal_node_keys_backward(f["grad_in"])
    tol = {"f32": 1e-6, "f16": 2e-2, "bf16": 6e-2}[dt]
    np.testing.assert_allclose(gk, f["grad_k"], atol=tol, rtol=tol)


@pytest.mark.parametrize("path", ADAPTER, ids=os.path.basename)
def test_oracle_adapter_matches_reference(path):
    f = np.load(path)
    dt = os.path.basename(path).split("_")[1]
    S = int(f["num_samples"])
    res = O.adapter_forward_backward(f["q"], f["k"], f["v"], f["grad_out"], f["gumbels"], S, dt)
    tol = {"f32": dict(out=5e-5, g=4e-4), "bf16": dict(out=2e-2, g=5e-2)}[dt]
    np.testing.assert_allclose(res["out"], f["out"], atol=tol["out"], rtol=tol["out"])
    for n in ("dq", "dk", "dv"):
        np.testing.assert_allclose(res[n], f[n], atol=tol["g"], rtol=tol["g"], err_msg=n)


CAUSAL = sorted(glob.glob(os.path.join(GOLDEN, "causal_*.npz")))
EXACT = sorted(glob.glob(os.path.join(GOLDEN, "exact_*.npz")))


def test_causal_fixtures_present():
    assert len(CAUSAL) == 4 and len(EXACT) == 4


@pytest.mark.parametrize("path", CAUSAL, ids=os.path.basename)
def test_oracle_causal_matches_reference(path):
    import torch

    from oracle import tree_oracle_torch as OT

    f = np.load(path)
    L, B, H, D, S = (int(x) for x in f["shape"])
    q, k, v, g = (_heads(f[n], H) for n in ("q", "k", "v", "grad_out"))
    res = O.causal_attention(q, k, v, f["gumbels"], S)
    np.testing.assert_allclose(res["out"].reshape(L, B, -1), f["out"], atol=5e-5, rtol=5e-5)
    np.testing.assert_allclose(res["weights"], f["weights"], atol=5e-5, rtol=5e-5)
    # the torch restatement reproduces outputs and the reference's autograd gradients
    qt, kt, vt = (torch.tensor(x, requires_grad=True) for x in (q, k, v))
    out, w, leaf = OT.causal_attention(qt, kt, vt, torch.tensor(f["gumbels"]), S)
    np.testing.assert_array_equal(leaf.numpy(), res["leaf"])
    out.backward(torch.tensor(g))
    np.testing.assert_allclose(out.detach().numpy().reshape(L, B, -1), f["out"], atol=5e-5, rtol=5e-5)
    for name, t in (("dq", qt), ("dk", kt), ("dv", vt)):
        np.testing.assert_allclose(t.grad.numpy().reshape(f[name].shape), f[name], atol=2e-4,
                                   rtol=2e-4, err_msg=name)


@pytest.mark.parametrize("path", EXACT, ids=os.path.basename)
def test_oracle_exact_matches_reference(path):
    import torch

    from oracle import tree_oracle_torch as OT

    f = np.load(path)
    L, B, H, D = (int(x) for x in f["shape"])
    causal = "causal" in os.path.basename(path)
    q, k, v, g = (_heads(f[n], H) for n in ("q", "k", "v", "grad_out"))
    out, w = O.deterministic_attention(q, k, v, causal)
    np.testing.assert_allclose(out.reshape(L, B, -1), f["out"], atol=5e-5, rtol=5e-5)
    np.testing.assert_allclose(w, f["weights"], atol=5e-5, rtol=5e-5)
    qt, kt, vt = (torch.tensor(x, requires_grad=True) for x in (q, k, v))
    ot, _ = OT.deterministic_attention(qt, kt, vt, causal)
    ot.backward(torch.tensor(g))
    for name, t in (("dq", qt), ("dk", kt), ("dv", vt)):
        np.testing.assert_allclose(t.grad.numpy().reshape(f[name].shape), f[name], atol=2e-4,
                                   rtol=2e-4, err_msg=name)


def test_tree_layout_nodes_summarise_their_subtrees():
    # float32 leaves whose halving steps are exact: node (d, i) = (mean L - mean R) / 2
    rng = np.random.default_rng(3)
    S = 64
    k = rng.integers(-8, 8, size=(S, 1, 2, 4)).astype(np.float32)
    nodes = O.tree_layout_node_keys(k, "f32")
    ln = 6
    for d in range(ln):
        span = S >> d
        for i in range(1 << d):
            lo = k[i * span:i * span + span // 2].mean(axis=0)
            hi = k[i * span + span // 2:(i + 1) * span].mean(axis=0)
            np.testing.assert_allclose(nodes[(1 << d) - 1 + i], (lo - hi) / 2, rtol=0, atol=1e-6)
    # a permutation of the reference array
    ref = O.haar_internal_node_keys(k, "f32")
    assert sorted(O.tree_layout_rows(S).tolist()) == list(range(S - 1))
    np.testing.assert_array_equal(np.sort(nodes.ravel()), np.sort(ref.ravel()))
