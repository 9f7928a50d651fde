"""Opt-in departures from the reference's semantics: the tree-correct node layout and
logit scaling by softmax_scale. Both are checked against the numpy oracle given torch's own
Gumbel draws for the same seed."""

import numpy as np
import pytest
import torch

import treeattn_b200 as ta
from oracle import tree_oracle as O
from treeattn_b200 import ops
from tests.test_gpu_parity import DEV, TORCH_DT, reference_gumbels

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("S,B,H,D", [(64, 1, 2, 32), (2048, 2, 3, 64), (16384, 1, 2, 128)])
def test_tree_layout_build_is_the_oracle_permutation(dtype, S, B, H, D):
    torch.manual_seed(S)
    k = torch.randn(S, B, H, D, device=DEV).to(TORCH_DT[dtype])
    got = ops.tree_build(k, node_layout="tree")
    want = O.tree_layout_node_keys(k.float().cpu().numpy(), dtype)
    np.testing.assert_array_equal(got.float().cpu().numpy(), want)
    # transpose: the gradient of sum(dk_int * nodes) w.r.t. the leaves
    dk_int = torch.randn(B, H, S - 1, D, device=DEV).permute(2, 0, 1, 3)
    dk = torch.empty(S, B, H, D, device=DEV)
    ops.tree_build_backward(dk_int, dk, "tree")
    rows = O.tree_layout_rows(S)
    want_dk = O.haar_internal_node_keys_backward(dk_int.cpu().numpy()[rows])
    np.testing.assert_allclose(dk.cpu().numpy(), want_dk, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("node_layout,scale_logits", [("tree", False), ("reference", True), ("tree", True)])
def test_options_end_to_end_against_oracle(node_layout, scale_logits):
    B, S, H, D, P = 1, 512, 2, 64, 8
    torch.manual_seed(11)
    q, k, v, go = (torch.randn(B, S, H, D, device=DEV) for _ in range(4))
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    torch.manual_seed(4)
    out = ta.tree_attention(qq, kk, vv, False, None, num_samples=P, node_layout=node_layout,
                            scale_logits=scale_logits)
    out.backward(go)
    torch.manual_seed(4)
    g = reference_gumbels((S, B, H, P, 2), O.log_n_of(S)).cpu().numpy()
    c = D ** -0.5 if scale_logits else 1.0
    f32 = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
    qs = (q * c).float() if scale_logits else q
    res = O.adapter_forward_backward(f32(qs), f32(k), f32(v), f32(go), g, P, "f32",
                                     node_layout=node_layout)
    np.testing.assert_allclose(f32(out), res["out"], atol=5e-5, rtol=0)
    np.testing.assert_allclose(f32(qq.grad), res["dq"] * c, atol=2e-4, rtol=2e-4)
    np.testing.assert_allclose(f32(kk.grad), res["dk"], atol=4e-4, rtol=4e-4)
    np.testing.assert_allclose(f32(vv.grad), res["dv"], atol=2e-4, rtol=2e-4)


def test_layouts_differ_and_bad_layout_raises():
    torch.manual_seed(0)
    k = torch.randn(256, 1, 1, 32, device=DEV)
    assert not torch.equal(ops.tree_build(k), ops.tree_build(k, node_layout="tree"))
    with pytest.raises(ValueError):
        ops.tree_build(k, node_layout="inorder")
