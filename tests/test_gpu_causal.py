"""GPU parity of the causal sampler (A9) and the exact mode (A10).

Mirrors treeattn-torch's causal / deterministic modes (treeattn_torch/_tree_mha.py:125-413),
checked against fixtures recorded from the reference (injected noise) and against the torch
restatement in oracle/ driven by torch's CUDA generator exactly as the reference draws.
"""

import glob
import os

import numpy as np
import pytest
import torch

import treeattn_b200 as ta
from oracle import tree_oracle as O
from oracle import tree_oracle_torch as OT
from tests.conftest import GOLDEN
from treeattn_b200 import autograd as AG
from treeattn_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"
CAUSAL = sorted(glob.glob(os.path.join(GOLDEN, "causal_*.npz")))
EXACT = sorted(glob.glob(os.path.join(GOLDEN, "exact_*.npz")))


def _t(x, dt=torch.float32):
    return torch.as_tensor(np.asarray(x)).to(device=DEV, dtype=dt)


def _heads(x, H):
    return x.reshape(x.shape[0], x.shape[1], H, -1)


@pytest.mark.parametrize("path", CAUSAL, ids=os.path.basename)
def test_causal_matches_reference_fixtures(path):
    f = np.load(path)
    L, B, H, D, S = (int(x) for x in f["shape"])
    q, k, v, go = (_t(_heads(f[n], H)) for n in ("q", "k", "v", "grad_out"))
    out = torch.empty_like(q)
    G = _t(f["gumbels"])
    if L > S:
        ops.exact_forward(q[:S], k, v, True, 0, out=out[:S], want_weights=False)
        _, st = ops.causal_forward(q[S:], k, v, S, S, out=out[S:], gumbels=G)
    else:
        _, st = ops.causal_forward(q, k, v, S, 0, out=out, gumbels=G)
    np.testing.assert_allclose(out.reshape(L, B, -1).cpu().numpy(), f["out"], atol=5e-5, rtol=5e-5)
    np.testing.assert_allclose(st.weights.cpu().numpy(), f["weights"], atol=5e-5, rtol=5e-5)
    dq = torch.empty_like(q)
    dk = torch.empty(k.shape, device=DEV)
    dv = torch.empty(v.shape, device=DEV)
    AG._causal_bwd(q, k, v, go, st, S, dq, dk, dv)
    np.testing.assert_allclose(dq.reshape(L, B, -1).cpu().numpy(), f["dq"], atol=2e-4, rtol=2e-4)
    np.testing.assert_allclose(dk.reshape(L - 1, B, -1).cpu().numpy(), f["dk"], atol=4e-4, rtol=4e-4)
    np.testing.assert_allclose(dv.reshape(L, B, -1).cpu().numpy(), f["dv"], atol=2e-4, rtol=2e-4)


@pytest.mark.parametrize("path", EXACT, ids=os.path.basename)
def test_exact_matches_reference_fixtures(path):
    f = np.load(path)
    L, B, H, D = (int(x) for x in f["shape"])
    causal = "causal" in os.path.basename(path)
    q, k, v = (_t(f[n]).requires_grad_(True) for n in ("q", "k", "v"))
    out, w = ta.hierarchical_attention(q, k, v, num_heads=H, is_causal=causal, mode="deterministic")
    out.backward(_t(f["grad_out"]))
    np.testing.assert_allclose(out.detach().cpu().numpy(), f["out"], atol=5e-5, rtol=5e-5)
    np.testing.assert_allclose(w.cpu().numpy(), f["weights"], atol=5e-5, rtol=5e-5)
    for name, t in (("dq", q), ("dk", k), ("dv", v)):
        np.testing.assert_allclose(t.grad.cpu().numpy(), f[name], atol=2e-4, rtol=2e-4, err_msg=name)


def reference_causal_gumbels(lsto, log_n, B, H, S):
    """The reference's draws: one (B,H,S,2) exponential_() per sampled query and level."""
    return torch.stack([
        torch.stack([torch.empty((B, H, S, 2), device=DEV).exponential_().log_().neg_()
                     for _ in range(log_n)]) for _ in range(lsto)])


@pytest.mark.parametrize("L,B,H,D,S", [(8, 1, 2, 16, 8), (64, 2, 2, 32, 4), (128, 1, 3, 64, 8),
                                       (256, 2, 2, 32, 16)])
def test_causal_generator_stream_and_gradients(L, B, H, D, S):
    E = H * D
    torch.manual_seed(77)
    q = torch.randn(L, B, E, device=DEV, requires_grad=True)
    k = torch.randn(L - 1, B, E, device=DEV, requires_grad=True)
    v = torch.randn(L, B, E, device=DEV, requires_grad=True)
    go = torch.randn(L, B, E, device=DEV)
    torch.manual_seed(0)
    out, w = ta.hierarchical_attention(q, k, v, num_heads=H, is_causal=True, num_samples=S)
    out.backward(go)
    torch.manual_seed(0)
    lsto = L - S if L > S else L
    G = reference_causal_gumbels(lsto, O.log_n_of(L), B, H, S).cpu()
    qc, kc, vc = (x.detach().cpu().reshape(x.shape[0], B, H, D).requires_grad_(True) for x in (q, k, v))
    ro, rw, rleaf = OT.causal_attention(qc, kc, vc, G, S)
    ro.backward(go.cpu().reshape(L, B, H, D))
    np.testing.assert_allclose(out.detach().cpu().numpy(), ro.detach().reshape(L, B, E).numpy(), atol=5e-5, rtol=5e-5)
    np.testing.assert_allclose(w.cpu().numpy(), rw.detach().numpy(), atol=5e-5, rtol=5e-5)
    for name, t, r in (("dq", q, qc), ("dk", k, kc), ("dv", v, vc)):
        np.testing.assert_allclose(t.grad.cpu().numpy(), r.grad.reshape(t.shape).numpy(), atol=4e-4,
                                   rtol=4e-4, err_msg=name)


@pytest.mark.parametrize("dtype,tol", [("bf16", 2e-2), ("f16", 5e-3)])
def test_causal_bshd_adapter_low_precision(dtype, tol):
    dt = {"bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    B, S, H, D, P = 1, 256, 2, 64, 8
    torch.manual_seed(3)
    scale = 0.5 if dtype == "f16" else 1.0
    q, k, v, go = (torch.randn(B, S, H, D, device=DEV).mul(scale).to(dt) for _ in range(4))
    qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
    torch.manual_seed(4)
    out = ta.tree_attention(qq, kk, vv, True, None, num_samples=P)
    out.backward(go)
    torch.manual_seed(4)
    G = reference_causal_gumbels(S - P, O.log_n_of(S), B, H, P).cpu()
    f32 = lambda t: t.detach().float().cpu()  # noqa: E731
    k_int = torch.tensor(O.haar_internal_node_keys(f32(k).transpose(0, 1).numpy(), dtype)).requires_grad_(True)
    qc = f32(q).transpose(0, 1).contiguous().requires_grad_(True)
    vc = f32(v).transpose(0, 1).contiguous().requires_grad_(True)
    ro, _, _ = OT.causal_attention(qc, k_int, vc, G, P)
    ro.backward(f32(go).transpose(0, 1))
    np.testing.assert_allclose(f32(out).numpy(), ro.detach().transpose(0, 1).numpy(), atol=tol, rtol=0)
    dk_leaf = O.haar_internal_node_keys_backward(k_int.grad.numpy())
    np.testing.assert_allclose(f32(qq.grad).numpy(), qc.grad.transpose(0, 1).numpy(), atol=2 * tol, rtol=tol)
    np.testing.assert_allclose(f32(vv.grad).numpy(), vc.grad.transpose(0, 1).numpy(), atol=2 * tol, rtol=tol)
    np.testing.assert_allclose(f32(kk.grad).numpy(), np.transpose(dk_leaf, (1, 0, 2, 3)), atol=2 * tol, rtol=tol)


def test_exact_generic_shapes_and_determinism():
    torch.manual_seed(5)
    for (L, N, B, H, D) in [(40, 64, 2, 3, 32), (16, 1024, 1, 2, 128)]:
        for causal in (False, True):
            q = torch.randn(L, B, H * D, device=DEV, requires_grad=True)
            k = torch.randn(N - 1, B, H * D, device=DEV, requires_grad=True)
            v = torch.randn(N, B, H * D, device=DEV, requires_grad=True)
            go = torch.randn(L, B, H * D, device=DEV)
            out, w = ta.hierarchical_attention(q, k, v, num_heads=H, is_causal=causal, mode="deterministic")
            out.backward(go)
            g1 = [t.grad.clone() for t in (q, k, v)]
            qc, kc, vc = (x.detach().cpu().reshape(x.shape[0], B, H, D).requires_grad_(True) for x in (q, k, v))
            ro, rw = OT.deterministic_attention(qc, kc, vc, causal)
            ro.backward(go.cpu().reshape(L, B, H, D))
            np.testing.assert_allclose(out.detach().cpu().numpy(), ro.detach().reshape(L, B, -1).numpy(), atol=1e-4, rtol=1e-4)
            for t, r in ((q, qc), (k, kc), (v, vc)):
                np.testing.assert_allclose(t.grad.cpu().numpy(), r.grad.reshape(t.shape).numpy(), atol=5e-4, rtol=5e-4)
            for t in (q, k, v):
                t.grad = None
            out2, _ = ta.hierarchical_attention(q, k, v, num_heads=H, is_causal=causal, mode="deterministic")
            out2.backward(go)
            for a, t in zip(g1, (q, k, v)):
                assert torch.equal(a, t.grad)
            for t in (q, k, v):
                t.grad = None
