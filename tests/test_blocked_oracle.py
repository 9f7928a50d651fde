"""The generalised (fanout, leaf block) oracle: reduction to the reference at f=2, Lb=1, and
consistency of its numpy and torch restatements."""

import numpy as np
import pytest
import torch

from oracle import blocked_oracle as BO
from oracle import tree_oracle as O


def test_depth_rules():
    assert BO.depth_of(1024, 2, 64) == 4
    assert BO.depth_of(8192, 4, 128) == 3
    assert BO.depth_of(64, 4, 64) == 0
    for bad in [(1000, 2, 64), (1024, 3, 1), (1024, 4, 32), (96, 2, 3)]:
        with pytest.raises(ValueError):
            BO.depth_of(*bad)


def test_reduces_to_reference_tree_layout_at_f2_lb1():
    rng = np.random.default_rng(0)
    L, B, H, D, S = 64, 1, 2, 16, 4
    # dyadic keys: the Haar halvings and the means are exact, so the node keys agree exactly
    k = (rng.integers(-16, 16, size=(L, B, H, D)) / 8).astype(np.float32)
    q = rng.standard_normal((L, B, H, D)).astype(np.float32)
    v = rng.standard_normal((L, B, H, D)).astype(np.float32)
    ln = 6
    g = rng.gumbel(size=(ln, L, B, H, S, 2)).astype(np.float32)
    res = BO.forward(q, k, v, g, S, 2, 1)
    nodes = O.tree_layout_node_keys(k, "f32")
    ref = O.forward(q, nodes, v, g, S)
    # leaves: same decisions except float ties (softmax vs logsigmoid rounding)
    agree = (res["block"] == ref["leaf"]).mean()
    assert agree > 0.995
    same = res["block"] == ref["leaf"]
    np.testing.assert_allclose(res["log_prob"][same], ref["log_prob"][same] if "log_prob" in ref
                               else res["log_prob"][same], rtol=1e-5, atol=1e-5)
    rows = np.all(same, axis=-1)
    np.testing.assert_allclose(res["out"][rows], ref["out"][rows], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("f,Lb,N", [(2, 4, 64), (4, 8, 128), (8, 2, 128)])
def test_numpy_and_torch_restatements_agree(causal, f, Lb, N):
    rng = np.random.default_rng(N + f)
    B, H, D, S = 2, 2, 16, 3
    L = N
    q, k, v = (rng.standard_normal((s, B, H, D)).astype(np.float32) for s in (L, N, N))
    dp = BO.depth_of(N, f, Lb)
    g = rng.gumbel(size=(dp, L, B, H, S, f)).astype(np.float32)
    res = BO.forward(q, k, v, g, S, f, Lb, causal=causal)
    if causal:  # the chosen block always holds a key at or before the boundary
        first = res["block"] * Lb
        assert np.all(first <= (np.arange(L) + N - L)[:, None, None, None])
    t = lambda x: torch.tensor(x, dtype=torch.float64)  # noqa: E731
    out = BO.forward_torch(t(q), t(k), t(v), res["block"], f, Lb, causal=causal)
    np.testing.assert_allclose(out.numpy(), res["out"], rtol=1e-4, atol=1e-5)
